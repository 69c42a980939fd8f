// tc_linear.cu -- online-dequant linear on the 5th-generation tensor cores.
//
// y[M, oc] = x[M, ic] . decode(W)^T with W in one of the reference's packed
// layouts, read in place (no load-time re-layout):
//   SPFP2  block_fp2_emu.py:231-267: per 16 weights, mantissa words m0, m1
//          (u16 LE, code i at bits 2i) then one byte e0 | e1 << 4;
//   FP3    fp3_emu.py:107-139: 8 codes of 3 bits in 3 bytes (code i at bit
//          3i), plus one e4m3 scale per 16 weights;
//   NVFP4  nvfp4_emu.py:81-107: two e2m1 codes per byte (even element in the
//          low nibble), plus one e4m3 scale per 16 weights.
// Every decoded weight is exact in bf16 (SPFP2: +-2^(e-10); FP3 / NVFP4: a
// code value with at most 2 significant bits times an e4m3 scale with 4), so
// the tensor core multiplies the caller's bf16 x by the exact weights.
//
// Work unit: 128 weight rows x 256 columns (TMA boxes of 128 rows of codes,
// and of scales),
// for one tile of N tokens; a job is all units of one (token tile, row
// block).  One CTA per SM.  Decode (M <= 16, N = 16) splits the units of all
// jobs evenly over the CTAs (stream-K): a CTA whose unit range starts or ends
// inside a job publishes a partial sum and, per 32-row slice, the last
// contributor adds them in CTA order, so the result does not depend on
// timing.  Prefill (N = 64, 128 or 256) hands whole jobs to the CTAs in turn.
//
// Roles inside a CTA (576 threads):
//   warps 0-15 decode: warp w works on TMEM lane quadrant w % 4 and on column
//              step w / 4 (64 columns) of every unit; thread r (mod 128) owns
//              weight row r of the row block = TMEM lane r.  Per step a thread
//              turns its packed bytes into 32 bf16x2 registers (SPFP2: prmt
//              table lookups; FP3 / NVFP4: a table of code pairs times the
//              block scale, one bf16x2 multiply per two weights) and stores
//              them to a TMEM A stage with one tcgen05.st.  After a job's last
//              unit the groups read the fp32 accumulators back with tcgen05.ld
//              (each a quarter of the tokens; warps 0-3 alone for 16-token
//              tiles), release them to the next job and write y.
//   warp 16    allocates TMEM; lane 0 issues tcgen05.mma (kind::f16, A from
//              TMEM, B = x from shared memory, D fp32 in TMEM) and commits
//              each stage back to its producer.
//   warp 17    lane 0 issues the TMA loads: weight tiles (before the
//              programmatic-launch wait, since weights never depend on the
//              previous kernel) and x tiles (128-byte swizzled, K-major).
//
// Every mbarrier wait is bounded (%globaltimer, 2 s); an expired wait records
// an error in the workspace word and the thread leaves its loop, so the CTA
// still reaches the final barrier and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace spark {
namespace tc {

constexpr int kRows = 128;            // weight rows per unit = MMA M = TMEM lanes
constexpr int kUnitCols = 256;        // columns per unit
constexpr int kSub = 4;               // 64-column sub-steps per unit (one A stage each)

// Packed bytes of one row in one unit: codes (SPFP2 16 pairs x 5 B, FP3
// 32 x 3 B, NVFP4 128 x 1 B) and e4m3 scales (16 per unit).
template <int FMT>
struct Wfmt {
    // 2:4 rows take 7 bytes per 32 weights: a 512-column unit (112 bytes) is
    // the smallest whole 16-byte TMA box; the other formats use 256 columns
    static constexpr int kSub = FMT == SPARK_FMT_TWOFOUR ? 8 : 4;      // 64-column steps per unit
    static constexpr int kCols = 64 * kSub;
    static constexpr int kCodeBytes =
        FMT == SPARK_FMT_SPFP2 ? 80 : (FMT == SPARK_FMT_FP3 ? 96 : (FMT == SPARK_FMT_NVFP4 ? 128 : 112));
    static constexpr int kScaleBytes = (FMT == SPARK_FMT_FP3 || FMT == SPARK_FMT_NVFP4) ? 16 : 0;
    static constexpr int kStageBytes = kRows * (kCodeBytes + kScaleBytes);   // multiple of 1024
    static constexpr bool kSwizzle = FMT == SPARK_FMT_NVFP4;                 // 128-byte rows: swizzle them
};
constexpr int kDecThreads = 512;      // 16 decode warps: four per TMEM lane quadrant
constexpr int kMmaWarp = 16;
constexpr int kProducerWarp = 17;
constexpr int kThreads = 576;
constexpr uint64_t kWaitNs = 2000000000ull;

template <int FMT, int N>
struct Cfg {
    using W = Wfmt<FMT>;
    // Weight tiles decode fast: a few stages ahead suffice.  x tiles come from
    // L2 and feed the tensor core directly, so big token tiles get the room
    // (256-token tiles: 4 + 4 measured ~2% faster than 3 weight + 5 x stages).
    static constexpr int kWStages = N >= 256 ? 4 : (N >= 128 ? 3 : 6);
    // A stages (64 columns each) and the D buffers share the CTA's TMEM.
    static constexpr int kAStages = N == 16 ? 12 : 8;
    static constexpr int kDBuf = N <= 128 ? 2 : 1;
    // Independent accumulators per D buffer: MMA kk of every 64-column step
    // adds into chain kk % kChains, so small-N MMAs do not wait on one
    // another's accumulator; the epilogue sums the chains (fixed order).
    static constexpr int kChains = N == 16 ? 4 : (N == 64 ? 2 : 1);
    static constexpr int kDStride = kChains * N;         // columns of one D buffer
    // decode groups that drain D after a job (each a slice of the N columns)
    static constexpr int kEpiGroups = N >= 64 ? 4 : 1;
    static constexpr int kDCols = kDBuf * kDStride;
    static constexpr uint32_t kTmemCols = kDCols + kAStages * 32 <= 256 ? 256u : 512u;
    // x tiles are small for decode-sized token tiles and latency-bound from
    // L2: keep many in flight
    // Up to 64 tokens one TMA brings a whole unit of x (kSub sub-tiles of N
    // rows x 64 columns, each 128-byte swizzled); larger tiles take one TMA per
    // 64-column sub-tile.
    static constexpr bool kXUnit = N <= 64;
    static constexpr int kXBytes = N * 128;                  // one sub-tile: N rows x 64 bf16
    static constexpr int kXStageBytes = kXUnit ? W::kSub * kXBytes : kXBytes;
    static constexpr int kXStages = kXUnit ? (N == 16 ? 8 : (W::kSub == 8 ? 2 : 3)) : (N == 128 ? 10 : (N == 256 ? 4 : 5));
    // dynamic shared memory (offsets from a 1024-aligned base)
    static constexpr int kX = 0;
    static constexpr int kW = kX + kXStages * kXStageBytes;
    static constexpr int kLut = kW + kWStages * W::kStageBytes;
    static constexpr int kTfCodes = kLut + 256 * 16;            // 2:4 code table (64 B)
    static constexpr int kBar = kTfCodes + 128;
    static constexpr int kNumBars = 2 * kWStages + 2 * kXStages + 2 * kAStages + 2 * kDBuf;
    static constexpr int kBytes = kBar + kNumBars * 8 + 16;
    static constexpr int kAlloc = kBytes + 1024;             // slack for aligning the base
    static_assert(kAlloc <= 232448, "shared memory above the 227 KB a CTA may use");
    static_assert(W::kStageBytes % 1024 == 0 && kXBytes % 1024 == 0, "stages must stay 1024-aligned");
};

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity to complete; false after kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t deadline = globaltimer_ns() + kWaitNs;
    while (!mbar_try(bar, parity))
        if (globaltimer_ns() > deadline) return false;
    return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            dst),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16, M = 128, no lanes disabled
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Instruction descriptor: D f32, A and B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset); the leading byte offset is unused
// for swizzled K-major layouts and set to 16 bytes.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3fffu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// ------------------------------------------------------------------ SPFP2 decode
// lut[b] for an exponent byte b = e0 | e1 << 4: {x0, y0, x1, y1} where, for a
// block exponent e and E = 117 + e the bf16 biased exponent of 2^(e-10),
// x = bytes [E >> 1, (E >> 1) | 0x80, 0, 0] (high bytes of +w, -w, 0, 0 for
// codes 0..3, block_fp2_emu.py:36) and y = bytes [(E & 1) << 7, same, 0, 0].
__device__ __forceinline__ uint2 exp_tables(uint32_t e) {
    const uint32_t E = 117u + e;
    return make_uint2((E >> 1) * 0x101u + 0x8000u, ((E & 1u) << 7) * 0x101u);
}

// Eight codes of one block -> four bf16x2 registers.  With selectors se
// (codes 0,1,4,5) and so (codes 2,3,6,7), see decode_pair, the output is in
// natural column order.
__device__ __forceinline__ void decode8(uint32_t se, uint32_t so, uint32_t tx, uint32_t ty, uint32_t* A) {
    const uint32_t he = prmt(tx, 0u, se), ho = prmt(tx, 0u, so);
    const uint32_t le = prmt(ty, 0u, se), lo = prmt(ty, 0u, so);
    A[0] = prmt(le, he, 0x5140u);
    A[1] = prmt(lo, ho, 0x5140u);
    A[2] = prmt(le, he, 0x7362u);
    A[3] = prmt(lo, ho, 0x7362u);
}

// One pair (16 weights): mantissa word mw = m0 | m1 << 16 (code i of a block
// at bits 2i), exponent tables t.  Swapping codes 1<->2 of every byte makes
// the nibble selectors (w & 0x3333) and (w >> 2 & 0x3333) pick codes
// (0,1,4,5) and (2,3,6,7), which decode8 interleaves into columns 0..7.
__device__ __forceinline__ void decode_pair(uint32_t mw, uint4 t, uint32_t* A) {
    const uint32_t inner = ((mw << 2) & 0x30303030u) | ((mw >> 2) & 0x0c0c0c0cu);
    const uint32_t w = (mw & 0xc3c3c3c3u) | inner;
    const uint32_t se = w & 0x33333333u, so = (w >> 2) & 0x33333333u;
    decode8(se, so, t.x, t.y, A);
    decode8(se >> 16, so >> 16, t.z, t.w, A + 4);
}

// 2:4 (two_four.py:112-189): a 7-byte pair holds two 16-blocks; block slot s
// is the 28-bit field at bit 28s: four 4-bit modes (group g at bit 4g), two
// sign bits per group (bits 16 + 2g, 17 + 2g) and the exponent (bit 24).
// tf_codes[mode | s0 << 4 | s1 << 5] = the group's four SPFP2 codes (code i at
// bit 2i; 0 = +, 1 = -, 2 = zero), so a block becomes one 16-code mantissa
// word for decode_pair, with the same exponent for both of its 8-halves.
__device__ __forceinline__ uint32_t twofour_codes(uint32_t idx) {
    const uint32_t mode = idx & 15u, s0 = (idx >> 4) & 1u, s1 = (idx >> 5) & 1u;
    const int pa[6] = {0, 0, 0, 1, 1, 2}, pb[6] = {1, 2, 3, 2, 3, 3};
    uint32_t c = 0xaau;                                          // four zero codes
    auto put = [&](int pos, uint32_t neg) { c = (c & ~(3u << (2 * pos))) | (neg << (2 * pos)); };
    if (mode < 6) {
        put(pa[mode], s0);
        put(pb[mode], s1);
    } else if (mode >= 8 && mode <= 11) {
        put((int)mode - 8, s0);
    }
    return c;
}

// One 16-block (28-bit field f) -> 8 bf16x2 registers.
__device__ __forceinline__ void decode_twofour_block(uint32_t f, const uint4* lut, const uint8_t* tf_codes,
                                                     uint32_t* A) {
    uint32_t mw = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint32_t idx = ((f >> (4 * g)) & 15u) | (((f >> (16 + 2 * g)) & 3u) << 4);
        mw |= (uint32_t)tf_codes[idx] << (8 * g);
    }
    const uint32_t e = (f >> 24) & 15u;
    decode_pair(mw, lut[e | (e << 4)], A);
}

// ------------------------------------------------------------------ FP3 / NVFP4 decode
// Tables in shared memory: scale2[b] = the e4m3 byte b as bf16, in both halves
// (fp8 to bf16 is exact: at most 4 significant bits; NaN stays NaN);
// pairv[v] = the two code values of a code pair v as bf16x2 (low half = the
// even column).  FP3 codes: sign bit 2, magnitudes {0, .5, 1, 1.5}
// (fp3_emu.py:14); NVFP4 codes: sign bit 3, magnitudes {0, .5, 1, 1.5, 2, 3,
// 4, 6} (nvfp4_emu.py:17).
__device__ __forceinline__ uint32_t bf16_bits(float f) { return __float_as_uint(f) >> 16; }

__device__ __forceinline__ uint32_t code_value_bf16(int fmt, uint32_t c) {
    if (fmt == SPARK_FMT_FP3) return bf16_bits(0.5f * (float)(c & 3u)) | ((c & 4u) << 13);
    const uint32_t m = c & 7u;
    const float v = m < 4u ? 0.5f * (float)m : (float)(1u << ((m - 2u) >> 1)) * (m & 1u ? 1.5f : 1.0f);
    return bf16_bits(v) | ((c & 8u) << 12);
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// One 64-column step (j) of row r of a weight stage: the packed bytes
// (q, 5 / 6 / 8 words) and the step's four e4m3 scales (sc).
template <int FMT>
__device__ __forceinline__ void load_step(const uint8_t* stage, int r, int j, uint32_t* q, uint32_t& sc) {
    using WF = Wfmt<FMT>;
    if constexpr (FMT == SPARK_FMT_SPFP2) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(stage + r * WF::kCodeBytes) + 5 * j;
#pragma unroll
        for (int k = 0; k < 5; ++k) q[k] = src[k];
    } else if constexpr (FMT == SPARK_FMT_TWOFOUR) {
        // step j = two pairs = bytes [14j, 14j + 14) of the 112-byte row: the
        // five words from the word holding byte 14j
        const uint32_t* src = reinterpret_cast<const uint32_t*>(stage + r * 112) + (14 * j) / 4;
#pragma unroll
        for (int k = 0; k < 5; ++k) q[k] = src[k];
    } else if constexpr (FMT == SPARK_FMT_FP3) {
        const uint2* src = reinterpret_cast<const uint2*>(stage + r * 96 + 24 * j);
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const uint2 v = src[k];
            q[2 * k] = v.x;
            q[2 * k + 1] = v.y;
        }
    } else {
        // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + 16 * ((2 * j + h) ^ (r & 7)));
            q[4 * h] = v.x;
            q[4 * h + 1] = v.y;
            q[4 * h + 2] = v.z;
            q[4 * h + 3] = v.w;
        }
    }
    if constexpr (WF::kScaleBytes > 0)
        sc = reinterpret_cast<const uint32_t*>(stage + kRows * WF::kCodeBytes + r * 16)[j];
}

// 64 weights of one row -> 32 bf16x2 registers in natural column order.
template <int FMT>
__device__ __forceinline__ void decode_step(const uint32_t* q, uint32_t sc, const uint4* lut, const uint32_t* scale2,
                                            const uint32_t* pairv, uint32_t* A, int j = 0,
                                            const uint8_t* tf_codes = nullptr) {
    if constexpr (FMT == SPARK_FMT_TWOFOUR) {
        // 56-bit pairs at byte offset (14j) % 4 and + 7 of the five words
        const int b0 = (14 * j) % 4;                 // 0 or 2
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
            const int bit = 8 * (b0 + 7 * pp), wi = bit >> 5, off = bit & 31;
            const uint32_t lo = off ? __funnelshift_r(q[wi], q[wi + 1], off) : q[wi];
            const uint32_t hi = off ? __funnelshift_r(q[wi + 1], q[wi + 2], off) : q[wi + 1];
            decode_twofour_block(lo & 0x0fffffffu, lut, tf_codes, A + 16 * pp);
            decode_twofour_block(__funnelshift_r(lo, hi, 28) & 0x0fffffffu, lut, tf_codes, A + 16 * pp + 8);
        }
    } else if constexpr (FMT == SPARK_FMT_SPFP2) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t mw, eb;
            if (k == 0) { mw = q[0]; eb = q[1] & 0xffu; }
            else if (k == 1) { mw = __funnelshift_r(q[1], q[2], 8); eb = (q[2] >> 8) & 0xffu; }
            else if (k == 2) { mw = __funnelshift_r(q[2], q[3], 16); eb = (q[3] >> 16) & 0xffu; }
            else { mw = __funnelshift_r(q[3], q[4], 24); eb = q[4] >> 24; }
            decode_pair(mw, lut[eb], A + 8 * k);
        }
    } else if constexpr (FMT == SPARK_FMT_FP3) {
        // 64 codes = 192 bits; code pair k (columns 2k, 2k+1) at bit 6k
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            const int bit = 6 * k, wi = bit >> 5, off = bit & 31;
            const uint32_t v = (off <= 26 ? (q[wi] >> off) : __funnelshift_r(q[wi], q[wi + 1], off)) & 63u;
            A[k] = mul_bf16x2(pairv[v], scale2[(sc >> (8 * (k >> 3))) & 0xffu]);
        }
    } else {
        // 64 codes = 32 bytes; byte k holds columns 2k, 2k+1
#pragma unroll
        for (int k = 0; k < 32; ++k)
            A[k] = mul_bf16x2(pairv[(q[k >> 2] >> (8 * (k & 3))) & 0xffu], scale2[(sc >> (8 * (k >> 3))) & 0xffu]);
    }
}

// ------------------------------------------------------------------ kernel
struct Params {
    const void* bias;
    void* y;
    float* partials;      // stream-K: [2 * grid][N][128]
    int* counters;        // stream-K: [jobs][4], zero between calls
    int* err;
    int64_t oc, ldy;
    int M, n_rb, n_kc, jobs, units, grid, stream_k, bias_dtype, y_dtype;
};

__device__ __forceinline__ int unit_begin(int c, const Params& p) {
    return (int)(((int64_t)c * p.units) / p.grid);
}
// CTA that owns unit u (stream-K)
__device__ __forceinline__ int unit_owner(int u, const Params& p) {
    return (int)((((int64_t)u + 1) * p.grid - 1) / p.units);
}

// One segment: column blocks [ka, kb) of job `job` (= token tile * n_rb + row block).
struct Seg {
    int job, ka, kb;
};

// The segments of one CTA, identical for every role.  Stream-K: the CTA's
// contiguous unit range cut at job boundaries.  Job mode: whole jobs
// c, c + grid, c + 2 grid, ...
struct SegIter {
    int u, u1, job;
    __device__ SegIter(int c, const Params& p) : u(unit_begin(c, p)), u1(unit_begin(c + 1, p)), job(c) {}
    __device__ bool next(Seg& s, const Params& p) {
        if (p.stream_k) {
            if (u >= u1) return false;
            s.job = u / p.n_kc;
            s.ka = u - s.job * p.n_kc;
            const int e = min(u1, (s.job + 1) * p.n_kc);
            s.kb = e - s.job * p.n_kc;
            u = e;
            return true;
        }
        if (job >= p.jobs) return false;
        s.job = job;
        s.ka = 0;
        s.kb = p.n_kc;
        job += p.grid;
        return true;
    }
};

// Flattened (job, column block) sequence of one CTA, for the producer.
struct UnitIter {
    SegIter it;
    Seg s;
    int kc;
    __device__ UnitIter(int c, const Params& p) : it(c, p), kc(0) { s.kb = 0; }
    __device__ bool next(const Params& p, int& job, int& col_block) {
        while (kc >= s.kb) {
            if (!it.next(s, p)) return false;
            kc = s.ka;
        }
        job = s.job;
        col_block = kc++;
        return true;
    }
};

template <int FMT, int N>
__global__ void __launch_bounds__(kThreads, 1)
    k_tc_linear(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                const __grid_constant__ CUtensorMap xmap, const Params p) {
    using C = Cfg<FMT, N>;
    using WF = Wfmt<FMT>;
    constexpr int kWStages = C::kWStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t tmem_base_s;
    uint4* lut = reinterpret_cast<uint4*>(smem + C::kLut);                        // SPFP2
    uint32_t* scale2 = reinterpret_cast<uint32_t*>(smem + C::kLut);                // FP3 / NVFP4
    uint32_t* pairv = reinterpret_cast<uint32_t*>(smem + C::kLut + 1024);
    uint8_t* tf_codes = smem + C::kTfCodes;                                        // 2:4
    const uint32_t bar0 = smem_u32(smem + C::kBar);
    auto w_full = [&](int s) { return bar0 + 8u * s; };
    auto w_empty = [&](int s) { return bar0 + 8u * (kWStages + s); };
    auto x_full = [&](int s) { return bar0 + 8u * (2 * kWStages + s); };
    auto x_empty = [&](int s) { return bar0 + 8u * (2 * kWStages + C::kXStages + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * kWStages + 2 * C::kXStages + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * kWStages + 2 * C::kXStages + C::kAStages + s); };
    auto d_full = [&](int s) { return bar0 + 8u * (2 * kWStages + 2 * C::kXStages + 2 * C::kAStages + s); };
    auto d_empty = [&](int s) {
        return bar0 + 8u * (2 * kWStages + 2 * C::kXStages + 2 * C::kAStages + C::kDBuf + s);
    };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWStages; ++s) { mbar_init(w_full(s), 1); mbar_init(w_empty(s), kDecThreads); }
        for (int s = 0; s < C::kXStages; ++s) { mbar_init(x_full(s), 1); mbar_init(x_empty(s), 1); }
        for (int s = 0; s < C::kAStages; ++s) { mbar_init(a_full(s), kRows); mbar_init(a_empty(s), 1); }
        for (int s = 0; s < C::kDBuf; ++s) { mbar_init(d_full(s), 1); mbar_init(d_empty(s), kRows * C::kEpiGroups); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_map(&wmap);
        if constexpr (WF::kScaleBytes > 0) prefetch_map(&smap);
        prefetch_map(&xmap);
    }
    for (int i = threadIdx.x; i < 256; i += kThreads) {
        if constexpr (FMT == SPARK_FMT_SPFP2 || FMT == SPARK_FMT_TWOFOUR) {
            const uint2 a = exp_tables(i & 15), b = exp_tables(i >> 4);
            lut[i] = make_uint4(a.x, a.y, b.x, b.y);
            if (FMT == SPARK_FMT_TWOFOUR && i < 64) tf_codes[i] = (uint8_t)twofour_codes((uint32_t)i);
        } else {
            const uint32_t sb = bf16_bits(e4m3_to_f32((uint32_t)i));
            scale2[i] = sb | (sb << 16);
            const int bits = FMT == SPARK_FMT_FP3 ? 3 : 4;
            if (i < (1 << (2 * bits))) {
                const uint32_t lo = code_value_bf16(FMT, (uint32_t)i & ((1u << bits) - 1u));
                const uint32_t hi = code_value_bf16(FMT, (uint32_t)i >> bits);
                pairv[i] = lo | (hi << 16);
            }
        }
    }
    if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_base_s), C::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Every CTA holds its TMEM now: the next kernel in the stream may start.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t tbase = tmem_base_s;
    const uint32_t a_col0 = C::kDCols;
    bool ok = true;

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            UnitIter wi(cta, p), xi(cta, p);
            int iw = 0, job, kc;
            auto issue_w = [&](int i, int jb, int k) -> bool {
                const int s = i % kWStages;
                if (!mbar_wait(w_empty(s), ((i / kWStages) & 1) ^ 1)) return false;
                const uint32_t dst = smem_u32(smem + C::kW + s * WF::kStageBytes);
                mbar_expect_tx(w_full(s), WF::kStageBytes);
                tma_load_2d(dst, &wmap, k * WF::kCodeBytes, (jb % p.n_rb) * kRows, w_full(s));
                if constexpr (WF::kScaleBytes > 0)
                    tma_load_2d(dst + kRows * WF::kCodeBytes, &smap, k * WF::kScaleBytes, (jb % p.n_rb) * kRows,
                                w_full(s));
                return true;
            };
            while (ok && iw < kWStages && wi.next(p, job, kc)) ok = issue_w(iw++, job, kc);
            // x and everything after it may depend on the previous kernel
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int i = 0; ok && xi.next(p, job, kc); ++i) {
                const int tb = job / p.n_rb;
                if constexpr (C::kXUnit) {
                    // the unit's kSub sub-tiles in one box of the [chunk][row][64] view of x
                    const int s = i % C::kXStages;
                    ok = mbar_wait(x_empty(s), ((i / C::kXStages) & 1) ^ 1);
                    if (!ok) break;
                    mbar_expect_tx(x_full(s), C::kXStageBytes);
                    tma_load_3d(smem_u32(smem + C::kX + s * C::kXStageBytes), &xmap, 0, tb * N, kc * WF::kSub,
                                x_full(s));
                } else {
                    for (int j = 0; j < WF::kSub && ok; ++j) {
                        const int ix = i * WF::kSub + j, s = ix % C::kXStages;
                        ok = mbar_wait(x_empty(s), ((ix / C::kXStages) & 1) ^ 1);
                        if (!ok) break;
                        mbar_expect_tx(x_full(s), C::kXBytes);
                        tma_load_2d(smem_u32(smem + C::kX + s * C::kXBytes), &xmap, kc * WF::kCols + j * 64, tb * N,
                                    x_full(s));
                    }
                }
                int jb, k;
                if (ok && wi.next(p, jb, k)) ok = issue_w(iw++, jb, k);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(N);
            SegIter it(cta, p);
            Seg sg;
            int i = 0;
            for (int seg = 0; ok && it.next(sg, p); ++seg) {
                const int buf = seg % C::kDBuf;
                ok = mbar_wait(d_empty(buf), ((seg / C::kDBuf) & 1) ^ 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tbase + (uint32_t)(buf * C::kDStride);
                for (int kc = sg.ka; kc < sg.kb && ok; ++kc, ++i) {
                    const int su = i % C::kXStages;
                    if constexpr (C::kXUnit) {
                        ok = mbar_wait(x_full(su), (i / C::kXStages) & 1);
                        if (!ok) break;
                    }
                    for (int j = 0; j < WF::kSub; ++j) {
                        const int ia = i * WF::kSub + j, sa = ia % C::kAStages;
                        const int sx = C::kXUnit ? su : ia % C::kXStages;
                        ok = mbar_wait(a_full(sa), (ia / C::kAStages) & 1) &&
                             (C::kXUnit || mbar_wait(x_full(sx), (ia / C::kXStages) & 1));
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t xb = C::kXUnit ? smem_u32(smem + C::kX + su * C::kXStageBytes + j * C::kXBytes)
                                                      : smem_u32(smem + C::kX + sx * C::kXBytes);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_ts(d_tmem + (uint32_t)((kk % C::kChains) * N), tbase + a_col0 + (uint32_t)(sa * 32 + kk * 8),
                                   sdesc_sw128(xb + kk * 32), idesc,
                                   (kc == sg.ka && j == 0 && kk < C::kChains) ? 0u : 1u);
                        mma_commit(a_empty(sa));
                        if (!C::kXUnit) mma_commit(x_empty(sx));
                    }
                    if (C::kXUnit && ok) mma_commit(x_empty(su));
                }
                if (ok) mma_commit(d_full(buf));
            }
        }
    } else {
        // ------------------------------------------------------------ decode (+ epilogue in group 0)
        const int group = warp >> 2, quad = warp & 3;    // group = the 64-column step of each unit
        const int r = threadIdx.x & (kRows - 1);          // row in the block = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        SegIter it(cta, p);
        Seg sg;
        int i = 0;
        for (int seg = 0; ok && it.next(sg, p); ++seg) {
            for (int kc = sg.ka; kc < sg.kb && ok; ++kc, ++i) {
                const int sw = i % kWStages;
                ok = __all_sync(0xffffffffu, mbar_wait(w_full(sw), (i / kWStages) & 1));
                if (!ok) break;
                // this thread's 64-column steps j = group + 4t of row r
                const uint8_t* stage = smem + C::kW + sw * WF::kStageBytes;
                constexpr int kT = WF::kSub / 4;
                constexpr int kQ = FMT == SPARK_FMT_FP3 ? 6 : (FMT == SPARK_FMT_NVFP4 ? 8 : 5);
                uint32_t q[kT][kQ];
                uint32_t sc[kT];
#pragma unroll
                for (int t = 0; t < kT; ++t) {
                    sc[t] = 0u;
                    load_step<FMT>(stage, r, group + 4 * t, q[t], sc[t]);
                }
                mbar_arrive(w_empty(sw));
#pragma unroll
                for (int t = 0; t < kT; ++t) {
                    const int j = group + 4 * t;
                    const int ia = i * WF::kSub + j, sa = ia % C::kAStages;
                    if (!__all_sync(0xffffffffu, mbar_wait(a_empty(sa), ((ia / C::kAStages) & 1) ^ 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t A[32];
                    decode_step<FMT>(q[t], sc[t], lut, scale2, pairv, A, j, tf_codes);
                    tmem_st32(tbase + lane_addr + a_col0 + (uint32_t)(sa * 32), A);
                    tmem_st_wait();
                    tc_fence_before();
                    mbar_arrive(a_full(sa));
                }
            }
            if (!ok || group >= C::kEpiGroups) continue;

            // ---------------- epilogue: group g reads D columns [g*N/G, (g+1)*N/G)
            // (thread r = row r), frees D, then writes y
            const int buf = seg % C::kDBuf;
            ok = __all_sync(0xffffffffu, mbar_wait(d_full(buf), (seg / C::kDBuf) & 1));
            if (!ok) break;
            tc_fence_after();
            const int job = sg.job;
            const int rb = job % p.n_rb, tb = job / p.n_rb;
            const int64_t row = (int64_t)rb * kRows + r;
            const int m0 = tb * N;
            const int mcount = min(N, p.M - m0);
            const uint32_t d_addr = tbase + lane_addr + (uint32_t)(buf * C::kDStride);
            // 16 accumulator columns, summed over the chains
            auto ld_sum16 = [&](uint32_t addr, float* v) {
                tmem_ld16(addr, v);
#pragma unroll
                for (int ch = 1; ch < C::kChains; ++ch) {
                    float w[16];
                    tmem_ld16(addr + (uint32_t)(ch * N), w);
#pragma unroll
                    for (int t = 0; t < 16; ++t) v[t] += w[t];
                }
            };
            const float bias = (p.bias && row < p.oc) ? load_as_float(p.bias, p.bias_dtype, row) : 0.0f;
            if (sg.ka == 0 && sg.kb == p.n_kc) {
                constexpr int kCols = N / C::kEpiGroups;
                const int c0 = group * kCols;
                float v[kCols];
#pragma unroll
                for (int c = 0; c < kCols; c += 16) ld_sum16(d_addr + c0 + c, v + c);
                tc_fence_before();
                mbar_arrive(d_empty(buf));
                if (row < p.oc)
#pragma unroll
                    for (int t = 0; t < kCols; ++t)
                        if (c0 + t < mcount)
                            store_from_float(p.y, p.y_dtype, (int64_t)(m0 + c0 + t) * p.ldy + row, v[t] + bias);
            } else if constexpr (N <= 64) {
                // Partial sum (stream-K): each group publishes its 16-token slice;
                // per (slice, 32-row quadrant), the warp that arrives last over
                // all contributors adds every contributor's partial in CTA order
                // (the same order on every call).
                constexpr int kCols = N / C::kEpiGroups;
                static_assert(kCols == 16, "one 16-token slice per epilogue group");
                const int c0 = group * kCols;
                const int slot = 2 * cta + (seg == 0 ? 0 : 1);
                float* mine = p.partials + ((int64_t)slot * N + c0) * kRows + r;
                {
                    float v[16];
                    ld_sum16(d_addr + c0, v);
                    tc_fence_before();
                    mbar_arrive(d_empty(buf));
#pragma unroll
                    for (int t = 0; t < 16; ++t) __stcg(mine + t * kRows, v[t]);
                }
                __threadfence();
                __syncwarp();
                const int job_u0 = job * p.n_kc;
                const int cA = unit_owner(job_u0, p), cB = unit_owner(job_u0 + p.n_kc - 1, p);
                int* counter = p.counters + ((int64_t)job * C::kEpiGroups + group) * 4 + quad;
                int last = 0;
                if (lane == 0) last = atomic_add_acq_rel(counter, 1) == cB - cA;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    if (row < p.oc) {
                        float acc[16];
#pragma unroll
                        for (int t = 0; t < 16; ++t) acc[t] = 0.0f;
                        for (int cc = cA; cc <= cB; ++cc) {
                            const int sl = 2 * cc + (unit_begin(cc, p) >= job_u0 ? 0 : 1);
                            const float* src = p.partials + ((int64_t)sl * N + c0) * kRows + r;
                            float v[16];
#pragma unroll
                            for (int t = 0; t < 16; ++t) v[t] = c0 + t < mcount ? __ldcg(src + t * kRows) : 0.0f;
#pragma unroll
                            for (int t = 0; t < 16; ++t) acc[t] += v[t];
                        }
#pragma unroll
                        for (int t = 0; t < 16; ++t)
                            if (c0 + t < mcount)
                                store_from_float(p.y, p.y_dtype, (int64_t)(m0 + c0 + t) * p.ldy + row, acc[t] + bias);
                    }
                    if (lane == 0) *counter = 0;
                }
            }
        }
    }
    if (!ok) report_device_error(p.err, 3);
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, C::kTmemCols);
    }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_mu;

int get_encoder() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode) return SPARK_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return set_error(SPARK_ERR_DEVICE, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return SPARK_OK;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SPARK_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SPARK_OK;
}

int sm_count_cached(int dev) {
    static int cnt[64] = {};
    if (dev < 0 || dev >= 64) return 148;
    if (!cnt[dev]) cudaDeviceGetAttribute(&cnt[dev], cudaDevAttrMultiProcessorCount, dev);
    return cnt[dev] > 0 ? cnt[dev] : 148;
}

template <int FMT, int N>
int launch(const CUtensorMap& wmap, const CUtensorMap& smap, const CUtensorMap& xmap, Params p, cudaStream_t s) {
    using Cf = Cfg<FMT, N>;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        static bool done[64] = {};
        std::lock_guard<std::mutex> lk(g_mu);
        if (!done[dev]) {
            cudaError_t e =
                cudaFuncSetAttribute(k_tc_linear<FMT, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kAlloc);
            if (e != cudaSuccess) return set_error((int)e, "k_tc_linear attribute: %s", cudaGetErrorString(e));
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cf::kAlloc;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_tc_linear<FMT, N>, wmap, smap, xmap, p);
    if (e != cudaSuccess) return set_error((int)e, "k_tc_linear launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

template <int FMT>
int launch_n(int N, const CUtensorMap& wmap, const CUtensorMap& smap, const CUtensorMap& xmap, const Params& p,
             cudaStream_t s) {
    switch (N) {
        case 16: return launch<FMT, 16>(wmap, smap, xmap, p, s);
        case 64: return launch<FMT, 64>(wmap, smap, xmap, p, s);
        case 128: return launch<FMT, 128>(wmap, smap, xmap, p, s);
        case 192: return launch<FMT, 192>(wmap, smap, xmap, p, s);
        default: return launch<FMT, 256>(wmap, smap, xmap, p, s);
    }
}

// Tokens per tile.  Above 128 tokens: the tile of 128, 192 or 256 tokens that
// needs the fewest token-rows per CTA once whole jobs are dealt out in rounds,
// weighted by the per-flop cost of a narrower tile (the same decode feeds
// less MMA work: ~35% slower at 128 tokens, ~13% at 192).  A 2560-row layer at
// 2048 tokens: 160 jobs of 256 tokens take two rounds on 148 SMs, the second
// nearly empty; 220 jobs of 192 take the same two rounds with 25% less work
// per job.
int token_tile(int64_t M, int64_t n_rb, int ctas) {
    if (M <= 16) return 16;
    if (M <= 64) return 64;
    if (M <= 128) return 128;
    auto cost = [&](int64_t n, double per_flop) {
        return (double)((n_rb * ((M + n - 1) / n) + ctas - 1) / ctas) * (double)n * per_flop;
    };
    int best = 256;
    double c = cost(256, 1.0);
    if (cost(192, 1.13) < c) { best = 192; c = cost(192, 1.13); }
    if (cost(128, 1.4) < c) best = 128;
    return best;
}

}  // namespace tc

// Workspace bytes of the tcgen05 path beyond the error word and counters:
// two partial slots of N x 128 fp32 per CTA (stream-K runs for 16- and
// 64-token tiles).
size_t tc_partials_bytes(int dev, int64_t M) {
    const int64_t n = M <= 16 ? 16 : 64;
    return (size_t)2 * tc::sm_count_cached(dev) * n * tc::kRows * sizeof(float);
}

bool tc_linear_ok(int fmt, const void* wq, const void* scales, const void* x, int x_dtype, int64_t ic,
                  int64_t ldx) {
    if (fmt != SPARK_FMT_SPFP2 && fmt != SPARK_FMT_FP3 && fmt != SPARK_FMT_NVFP4 && fmt != SPARK_FMT_TWOFOUR)
        return false;
    if ((fmt == SPARK_FMT_FP3 || fmt == SPARK_FMT_NVFP4) && !aligned(scales, 16)) return false;
    const int64_t unit = fmt == SPARK_FMT_TWOFOUR ? 512 : 256;
    return x_dtype == SPARK_DTYPE_BF16 && ic % unit == 0 && aligned(wq, 16) && aligned(x, 16) && (ldx % 8) == 0;
}

// Linear through k_tc_linear (SPFP2, FP3 or NVFP4, reference layouts).
// `counters` must hold max_counters zero ints (up to 16 per job are used);
// `partials` tc_partials_bytes(dev, M) bytes.
int tc_linear(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int64_t M, int64_t oc, int64_t ic,
              int64_t ldx, const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy, int* err,
              int* counters, int64_t max_counters, float* partials, cudaStream_t s) {
    SPARK_REQUIRE(tc_linear_ok(fmt, wq, scales, x, SPARK_DTYPE_BF16, ic, ldx), SPARK_ERR_ALIGNMENT,
                  "tcgen05 path: SPFP2/FP3/NVFP4, ic %% 256, 16-byte aligned weights, scales and x, ldx %% 8");
    int rc = tc::get_encoder();
    if (rc) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    const int ctas = tc::sm_count_cached(dev);
    const int64_t unit_cols = fmt == SPARK_FMT_TWOFOUR ? 512 : 256;
    const int64_t n_rb = (oc + tc::kRows - 1) / tc::kRows, n_kc = ic / unit_cols;
    const int N = tc::token_tile(M, n_rb, ctas);
    const int64_t n_tb = (M + N - 1) / N;
    const int64_t jobs = n_rb * n_tb;
    SPARK_REQUIRE(16 * jobs <= max_counters, SPARK_ERR_UNSUPPORTED, "tcgen05 path: %lld jobs above %lld",
                  (long long)jobs, (long long)(max_counters / 16));
    const int64_t units = jobs * n_kc;
    SPARK_REQUIRE(units < (1ll << 31) / 1024, SPARK_ERR_UNSUPPORTED, "tcgen05 path: problem too large");
    const int code_bytes =
        fmt == SPARK_FMT_SPFP2 ? 80 : (fmt == SPARK_FMT_FP3 ? 96 : (fmt == SPARK_FMT_NVFP4 ? 128 : 112));
    const uint64_t row_code_bytes = (uint64_t)(ic / unit_cols * code_bytes);
    alignas(64) CUtensorMap wmap, smap, xmap;
    rc = tc::encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, row_code_bytes, (uint64_t)oc, row_code_bytes,
                       (uint32_t)code_bytes, tc::kRows,
                       fmt == SPARK_FMT_NVFP4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    if (fmt == SPARK_FMT_SPFP2 || fmt == SPARK_FMT_TWOFOUR) {
        smap = wmap;                      // unused
    } else {
        rc = tc::encode_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, scales, (uint64_t)(ic / 16), (uint64_t)oc,
                           (uint64_t)(ic / 16), 16, tc::kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    if (N <= 64) {
        // [ic/64 chunks][M rows][64 columns] view of x: one box = a unit's sub-tiles
        const cuuint64_t dims[3] = {64, (cuuint64_t)M, (cuuint64_t)(ic / 64)};
        const cuuint64_t strides[2] = {(cuuint64_t)ldx * 2, 128};
        const cuuint32_t box[3] = {64, (cuuint32_t)N, (cuuint32_t)(unit_cols / 64)};
        const cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = tc::g_encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(SPARK_ERR_INVALID, "cuTensorMapEncodeTiled (x, 3-d) failed (%d)", (int)r);
    } else {
        rc = tc::encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)ic, (uint64_t)M, (uint64_t)ldx * 2, 64,
                           (uint32_t)N, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    tc::Params p = {};
    p.bias = bias;
    p.y = y;
    p.partials = partials;
    p.counters = counters;
    p.err = err;
    p.oc = oc;
    p.ldy = ldy;
    p.M = (int)M;
    p.n_rb = (int)n_rb;
    p.n_kc = (int)n_kc;
    p.jobs = (int)jobs;
    p.units = (int)units;
    // Decode: units split evenly over the CTAs (stream-K, 16-token partials).
    // Larger token tiles: whole jobs in turn, no partial sums.
    p.stream_k = (N == 16 || (N == 64 && jobs < ctas)) ? 1 : 0;
    p.grid = (int)(p.stream_k ? std::min<int64_t>(units, ctas) : std::min<int64_t>(jobs, ctas));
    p.bias_dtype = bias_dtype;
    p.y_dtype = y_dtype;
    switch (fmt) {
        case SPARK_FMT_SPFP2: return tc::launch_n<SPARK_FMT_SPFP2>(N, wmap, smap, xmap, p, s);
        case SPARK_FMT_FP3: return tc::launch_n<SPARK_FMT_FP3>(N, wmap, smap, xmap, p, s);
        case SPARK_FMT_NVFP4: return tc::launch_n<SPARK_FMT_NVFP4>(N, wmap, smap, xmap, p, s);
        default: return tc::launch_n<SPARK_FMT_TWOFOUR>(N, wmap, smap, xmap, p, s);
    }
}

}  // namespace spark

// ====================================================================== chains
// One persistent launch over a list of dependent ops (a decode step of a
// layer stack): dequant linears with up to 16 tokens, and SiLU(gate) * up.
// Every CTA takes part in every op (stream-K over the op's units, as the
// single-op kernel does for 16-token tiles) and the stage rings run straight
// across op boundaries, so the weights of the next op stream and decode
// while the previous one finishes.  Op k is complete when its done counter
// reaches its target (each CTA's epilogue warps add one after writing their
// rows); an op that reads an earlier op's output waits, bounded, for that
// count before its x tiles are loaded.  The launch is cooperative: every CTA
// is resident, so the waits between CTAs always end.
namespace spark {
namespace tc {

constexpr int kMaxOps = 16;
constexpr int kCN = 16;                  // tokens per tile
constexpr int kCWStage = 18432;          // largest weight stage (NVFP4: 128 x (128 + 16) B)
constexpr int kCWStages = 6;
constexpr int kCXStages = 32;
constexpr int kCAStages = 12;
constexpr int kCChains = 4;
constexpr int kCDStride = kCChains * kCN;
constexpr int kCDCols = 2 * kCDStride;
constexpr uint32_t kCTmemCols = 512;
static_assert(kCDCols + kCAStages * 32 <= 512, "TMEM budget");
// dynamic shared memory
constexpr int kCX = 0;
constexpr int kCW = kCX + kCXStages * kCN * 128;
constexpr int kCLut = kCW + kCWStages * kCWStage;       // SPFP2 table (4 KB)
constexpr int kCScale = kCLut + 4096;                   // e4m3 -> bf16x2 (1 KB)
constexpr int kCPair3 = kCScale + 1024;                 // FP3 code pairs (256 B)
constexpr int kCPair4 = kCPair3 + 256;                  // NVFP4 code pairs (1 KB)
constexpr int kCBar = kCPair4 + 1024;
constexpr int kCNumBars = 2 * kCWStages + 2 * kCXStages + 2 * kCAStages + 4;
constexpr int kCAlloc = kCBar + kCNumBars * 8 + 16 + 1024;
static_assert(kCAlloc <= 232448, "chain kernel shared memory");

struct ChainOp {
    int kind;                // 0 linear, 1 silu_mul
    int fmt, dep0, dep1, target;
    int n_rb, n_kc, units, bias_dtype, y_dtype, stage_bytes;
    int64_t oc, ldy, n;      // n: silu element count
    const void* bias;
    void* y;
    const void* g;
    const void* u;
    float* partials;         // linear: [2 * grid][16][128]
    int* counters;           // linear: [n_rb][4]
};

struct ChainProgram {
    CUtensorMap wmap[kMaxOps], smap[kMaxOps], xmap[kMaxOps];
    ChainOp op[kMaxOps];
    int n_ops, grid, M;
    int* done;               // [kMaxOps], zero at launch
    int* err;
};

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait for an op's completion count; false after kWaitNs.
__device__ bool wait_done(const int* done, int k, int target) {
    if (k < 0 || ld_acquire(done + k) >= target) return true;
    const uint64_t deadline = globaltimer_ns() + kWaitNs;
    while (ld_acquire(done + k) < target) {
        if (globaltimer_ns() > deadline) return false;
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ int op_unit_begin(int c, int units, int grid) {
    return (int)(((int64_t)c * units) / grid);
}
__device__ __forceinline__ int op_unit_owner(int u, int units, int grid) {
    return (int)((((int64_t)u + 1) * grid - 1) / units);
}

// Units of the linear ops of a chain, for this CTA, in program order.
struct ChainUnits {
    const ChainProgram* pr;
    int cta, k, u, u1;
    __device__ ChainUnits(const ChainProgram& p, int c) : pr(&p), cta(c), k(-1), u(0), u1(0) {}
    // next (op, job, column block); false at the end
    __device__ bool next(int& op, int& job, int& kc) {
        while (u >= u1) {
            if (++k >= pr->n_ops) return false;
            const ChainOp& o = pr->op[k];
            if (o.kind != 0) { u = u1 = 0; continue; }
            u = op_unit_begin(cta, o.units, pr->grid);
            u1 = op_unit_begin(cta + 1, o.units, pr->grid);
        }
        op = k;
        job = u / pr->op[k].n_kc;
        kc = u - job * pr->op[k].n_kc;
        ++u;
        return true;
    }
};

template <int FMT>
__device__ __forceinline__ void decode_op_step(const uint8_t* stage, int r, int j, const uint4* lut,
                                               const uint32_t* scale2, const uint32_t* pair3, const uint32_t* pair4,
                                               uint32_t* A) {
    uint32_t q[FMT == SPARK_FMT_SPFP2 ? 5 : (FMT == SPARK_FMT_FP3 ? 6 : 8)];
    uint32_t sc = 0u;
    load_step<FMT>(stage, r, j, q, sc);
    decode_step<FMT>(q, sc, lut, scale2, FMT == SPARK_FMT_FP3 ? pair3 : pair4, A);
}

__global__ void __launch_bounds__(kThreads, 1) k_tc_chain(const __grid_constant__ ChainProgram pr) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t tmem_base_s;
    uint4* lut = reinterpret_cast<uint4*>(smem + kCLut);
    uint32_t* scale2 = reinterpret_cast<uint32_t*>(smem + kCScale);
    uint32_t* pair3 = reinterpret_cast<uint32_t*>(smem + kCPair3);
    uint32_t* pair4 = reinterpret_cast<uint32_t*>(smem + kCPair4);
    const uint32_t bar0 = smem_u32(smem + kCBar);
    auto w_full = [&](int s) { return bar0 + 8u * s; };
    auto w_empty = [&](int s) { return bar0 + 8u * (kCWStages + s); };
    auto x_full = [&](int s) { return bar0 + 8u * (2 * kCWStages + s); };
    auto x_empty = [&](int s) { return bar0 + 8u * (2 * kCWStages + kCXStages + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * kCWStages + 2 * kCXStages + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * kCWStages + 2 * kCXStages + kCAStages + s); };
    auto d_full = [&](int s) { return bar0 + 8u * (2 * kCWStages + 2 * kCXStages + 2 * kCAStages + s); };
    auto d_empty = [&](int s) { return bar0 + 8u * (2 * kCWStages + 2 * kCXStages + 2 * kCAStages + 2 + s); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kCWStages; ++s) { mbar_init(w_full(s), 1); mbar_init(w_empty(s), kDecThreads); }
        for (int s = 0; s < kCXStages; ++s) { mbar_init(x_full(s), 1); mbar_init(x_empty(s), 1); }
        for (int s = 0; s < kCAStages; ++s) { mbar_init(a_full(s), kRows); mbar_init(a_empty(s), 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(d_full(s), 1); mbar_init(d_empty(s), kRows); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < 256; i += kThreads) {
        const uint2 a = exp_tables(i & 15), b = exp_tables(i >> 4);
        lut[i] = make_uint4(a.x, a.y, b.x, b.y);
        const uint32_t sb = bf16_bits(e4m3_to_f32((uint32_t)i));
        scale2[i] = sb | (sb << 16);
        pair4[i] = code_value_bf16(SPARK_FMT_NVFP4, i & 15u) | (code_value_bf16(SPARK_FMT_NVFP4, i >> 4) << 16);
        if (i < 64) pair3[i] = code_value_bf16(SPARK_FMT_FP3, i & 7u) | (code_value_bf16(SPARK_FMT_FP3, i >> 3) << 16);
    }
    if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_base_s), kCTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base_s;
    const uint32_t a_col0 = kCDCols;
    bool ok = true;

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            ChainUnits wi(pr, cta), xi(pr, cta);
            int iw = 0, op, job, kc;
            auto issue_w = [&](int i, int o, int jb, int k) -> bool {
                const int s = i % kCWStages;
                if (!mbar_wait(w_empty(s), ((i / kCWStages) & 1) ^ 1)) return false;
                const ChainOp& c = pr.op[o];
                const uint32_t dst = smem_u32(smem + kCW + s * kCWStage);
                const int code_bytes = c.fmt == SPARK_FMT_SPFP2 ? 80 : (c.fmt == SPARK_FMT_FP3 ? 96 : 128);
                const int row = (jb % c.n_rb) * kRows;
                mbar_expect_tx(w_full(s), c.stage_bytes);
                tma_load_2d(dst, &pr.wmap[o], k * code_bytes, row, w_full(s));
                if (c.fmt != SPARK_FMT_SPFP2) tma_load_2d(dst + kRows * code_bytes, &pr.smap[o], k * 16, row, w_full(s));
                return true;
            };
            while (ok && iw < kCWStages && wi.next(op, job, kc)) ok = issue_w(iw++, op, job, kc);
            int cur = -1;
            for (int i = 0; ok && xi.next(op, job, kc); ++i) {
                const ChainOp& c = pr.op[op];
                if (op != cur) {
                    // the op's input comes from earlier ops: wait until they are complete
                    cur = op;
                    ok = wait_done(pr.done, c.dep0, c.dep0 >= 0 ? pr.op[c.dep0].target : 0) &&
                         wait_done(pr.done, c.dep1, c.dep1 >= 0 ? pr.op[c.dep1].target : 0);
                    if (!ok) break;
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                const int tb = job / c.n_rb;
                for (int j = 0; j < kSub && ok; ++j) {
                    const int ix = i * kSub + j, s = ix % kCXStages;
                    ok = mbar_wait(x_empty(s), ((ix / kCXStages) & 1) ^ 1);
                    if (!ok) break;
                    mbar_expect_tx(x_full(s), kCN * 128);
                    tma_load_2d(smem_u32(smem + kCX + s * kCN * 128), &pr.xmap[op], kc * kUnitCols + j * 64,
                                tb * kCN, x_full(s));
                }
                int o2, jb, k;
                if (ok && wi.next(o2, jb, k)) ok = issue_w(iw++, o2, jb, k);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kCN);
            int i = 0, seg = 0;
            for (int op = 0; ok && op < pr.n_ops; ++op) {
                const ChainOp& c = pr.op[op];
                if (c.kind != 0) continue;
                int u = op_unit_begin(cta, c.units, pr.grid);
                const int u1 = op_unit_begin(cta + 1, c.units, pr.grid);
                while (ok && u < u1) {
                    const int job = u / c.n_kc, ka = u - job * c.n_kc;
                    const int kb = min(c.n_kc, ka + (u1 - u));
                    const int buf = seg & 1;
                    ok = mbar_wait(d_empty(buf), ((seg >> 1) & 1) ^ 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t d_tmem = tbase + (uint32_t)(buf * kCDStride);
                    for (int kc = ka; kc < kb && ok; ++kc, ++i) {
                        for (int j = 0; j < kSub; ++j) {
                            const int ia = i * kSub + j, sa = ia % kCAStages, sx = ia % kCXStages;
                            ok = mbar_wait(a_full(sa), (ia / kCAStages) & 1) &&
                                 mbar_wait(x_full(sx), (ia / kCXStages) & 1);
                            if (!ok) break;
                            tc_fence_after();
                            const uint32_t xb = smem_u32(smem + kCX + sx * kCN * 128);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                mma_ts(d_tmem + (uint32_t)((kk % kCChains) * kCN),
                                       tbase + a_col0 + (uint32_t)(sa * 32 + kk * 8), sdesc_sw128(xb + kk * 32), idesc,
                                       (kc == ka && j == 0 && kk < kCChains) ? 0u : 1u);
                            mma_commit(a_empty(sa));
                            mma_commit(x_empty(sx));
                        }
                    }
                    if (ok) mma_commit(d_full(buf));
                    u += kb - ka;
                    ++seg;
                }
            }
        }
    } else {
        // ------------------------------------------------------------ decode, epilogue, SiLU ops
        const int group = warp >> 2, quad = warp & 3;
        const int r = threadIdx.x & (kRows - 1);
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        int i = 0, seg = 0;
        for (int op = 0; ok && op < pr.n_ops; ++op) {
            const ChainOp& c = pr.op[op];
            if (c.kind == 1) {
                // SiLU(gate) * up over this CTA's slice, once gate and up are complete
                if (lane == 0)
                    ok = wait_done(pr.done, c.dep0, pr.op[c.dep0].target) &&
                         wait_done(pr.done, c.dep1, pr.op[c.dep1].target);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                const int64_t e0 = (int64_t)cta * c.n / pr.grid, e1 = (int64_t)(cta + 1) * c.n / pr.grid;
                const __nv_bfloat16* g = static_cast<const __nv_bfloat16*>(c.g);
                const __nv_bfloat16* uu = static_cast<const __nv_bfloat16*>(c.u);
                __nv_bfloat16* o = static_cast<__nv_bfloat16*>(c.y);
                for (int64_t e = e0 + threadIdx.x; e < e1; e += kDecThreads) {
                    const float a = __bfloat162float(__ldcg(g + e)), b = __bfloat162float(__ldcg(uu + e));
                    o[e] = __float2bfloat16_rn(a / (1.0f + __expf(-a)) * b);
                }
                __syncwarp();
                if (lane == 0) red_release_add(pr.done + op, 1);
                continue;
            }
            int u = op_unit_begin(cta, c.units, pr.grid);
            const int u1 = op_unit_begin(cta + 1, c.units, pr.grid), cu0 = u;
            while (ok && u < u1) {
                const int job = u / c.n_kc, ka = u - job * c.n_kc;
                const int kb = min(c.n_kc, ka + (u1 - u));
                for (int kc = ka; kc < kb && ok; ++kc, ++i) {
                    const int sw = i % kCWStages;
                    ok = __all_sync(0xffffffffu, mbar_wait(w_full(sw), (i / kCWStages) & 1));
                    if (!ok) break;
                    const int ia = i * kSub + group, sa = ia % kCAStages;
                    const uint8_t* stage = smem + kCW + sw * kCWStage;
                    uint32_t A[32];
                    // read the stage before releasing it; decode after the A stage is free
                    uint32_t q[8];
                    uint32_t sc = 0u;
                    if (c.fmt == SPARK_FMT_SPFP2) load_step<SPARK_FMT_SPFP2>(stage, r, group, q, sc);
                    else if (c.fmt == SPARK_FMT_FP3) load_step<SPARK_FMT_FP3>(stage, r, group, q, sc);
                    else load_step<SPARK_FMT_NVFP4>(stage, r, group, q, sc);
                    mbar_arrive(w_empty(sw));
                    if (!__all_sync(0xffffffffu, mbar_wait(a_empty(sa), ((ia / kCAStages) & 1) ^ 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (c.fmt == SPARK_FMT_SPFP2) decode_step<SPARK_FMT_SPFP2>(q, sc, lut, scale2, pair3, A);
                    else if (c.fmt == SPARK_FMT_FP3) decode_step<SPARK_FMT_FP3>(q, sc, lut, scale2, pair3, A);
                    else decode_step<SPARK_FMT_NVFP4>(q, sc, lut, scale2, pair4, A);
                    tmem_st32(tbase + lane_addr + a_col0 + (uint32_t)(sa * 32), A);
                    tmem_st_wait();
                    tc_fence_before();
                    mbar_arrive(a_full(sa));
                }
                if (!ok) break;
                const int seg_first = u == cu0;
                u += kb - ka;
                const int buf = seg & 1;
                ++seg;
                if (group != 0) continue;

                // ---------------- epilogue of this segment (group 0, thread r = row r)
                ok = __all_sync(0xffffffffu, mbar_wait(d_full(buf), ((seg - 1) >> 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const int rb = job % c.n_rb, tb = job / c.n_rb;
                const int64_t row = (int64_t)rb * kRows + r;
                const int m0 = tb * kCN, mcount = min(kCN, pr.M - m0);
                const uint32_t d_addr = tbase + lane_addr + (uint32_t)(buf * kCDStride);
                float v[16];
                tmem_ld16(d_addr, v);
#pragma unroll
                for (int ch = 1; ch < kCChains; ++ch) {
                    float w[16];
                    tmem_ld16(d_addr + (uint32_t)(ch * kCN), w);
#pragma unroll
                    for (int t = 0; t < 16; ++t) v[t] += w[t];
                }
                tc_fence_before();
                mbar_arrive(d_empty(buf));
                const float bias = (c.bias && row < c.oc) ? load_as_float(c.bias, c.bias_dtype, row) : 0.0f;
                if (ka == 0 && kb == c.n_kc) {
                    if (row < c.oc)
#pragma unroll
                        for (int t = 0; t < 16; ++t)
                            if (t < mcount) store_from_float(c.y, c.y_dtype, (int64_t)(m0 + t) * c.ldy + row, v[t] + bias);
                    continue;
                }
                // partial sum: publish; the last contributor per 32-row quadrant adds them in CTA order
                const int slot = 2 * cta + (seg_first ? 0 : 1);
                float* mine = c.partials + (int64_t)slot * kCN * kRows + r;
#pragma unroll
                for (int t = 0; t < 16; ++t) __stcg(mine + t * kRows, v[t]);
                __syncwarp();
                const int job_u0 = job * c.n_kc;
                const int cA = op_unit_owner(job_u0, c.units, pr.grid);
                const int cB = op_unit_owner(job_u0 + c.n_kc - 1, c.units, pr.grid);
                int* counter = c.counters + job * 4 + quad;
                int last = 0;
                if (lane == 0) last = atomic_add_acq_rel(counter, 1) == cB - cA;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                if (row < c.oc) {
                    float acc[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t) acc[t] = 0.0f;
                    for (int cc = cA; cc <= cB; ++cc) {
                        const int sl = 2 * cc + (op_unit_begin(cc, c.units, pr.grid) >= job_u0 ? 0 : 1);
                        const float* src = c.partials + (int64_t)sl * kCN * kRows + r;
                        float w[16];
#pragma unroll
                        for (int t = 0; t < 16; ++t) w[t] = t < mcount ? __ldcg(src + t * kRows) : 0.0f;
#pragma unroll
                        for (int t = 0; t < 16; ++t) acc[t] += w[t];
                    }
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        if (t < mcount) store_from_float(c.y, c.y_dtype, (int64_t)(m0 + t) * c.ldy + row, acc[t] + bias);
                }
                if (lane == 0) *counter = 0;
            }
            if (!ok) break;
            // this CTA's rows of op are written (group 0 warps, one count each)
            if (group == 0) {
                __syncwarp();
                if (lane == 0) red_release_add(pr.done + op, 1);
            }
        }
    }
    if (!ok) report_device_error(pr.err, 4);
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tbase, kCTmemCols);
    }
}

}  // namespace tc
}  // namespace spark

// ---------------------------------------------------------------------- C ABI
using namespace spark;

extern "C" {

size_t spark_linear_chain_workspace_size(int n_ops) {
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t grid = (size_t)tc::sm_count_cached(dev);
    // error word, done counters, fixup counters (64 Ki), per-op partials
    return 512 + (size_t)65536 * 4 + (size_t)std::max(n_ops, 0) * 2 * grid * tc::kCN * tc::kRows * 4;
}

int spark_linear_chain(const SparkChainOp* ops, int n_ops, int64_t M, void* workspace, size_t workspace_bytes,
                       void* stream) {
    SPARK_REQUIRE(ops && n_ops >= 1 && n_ops <= tc::kMaxOps, SPARK_ERR_INVALID,
                  "spark_linear_chain: 1..%d ops", tc::kMaxOps);
    SPARK_REQUIRE(M >= 1 && M <= 16, SPARK_ERR_UNSUPPORTED, "spark_linear_chain: M must be 1..16");
    SPARK_REQUIRE(workspace && aligned(workspace, 256) && workspace_bytes >= spark_linear_chain_workspace_size(n_ops),
                  SPARK_ERR_WORKSPACE, "spark_linear_chain: workspace of %zu bytes (256-aligned) needed",
                  spark_linear_chain_workspace_size(n_ops));
    int rc = tc::get_encoder();
    if (rc) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = tc::sm_count_cached(dev);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    static tc::ChainProgram pr;                 // built on the host, copied into the launch
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    memset(&pr, 0, sizeof(pr));
    pr.n_ops = n_ops;
    pr.grid = grid;
    pr.M = (int)M;
    pr.err = reinterpret_cast<int*>(ws);
    pr.done = reinterpret_cast<int*>(ws + 256);
    int* counters = reinterpret_cast<int*>(ws + 512);
    int64_t counter_next = 0;
    float* partials = reinterpret_cast<float*>(ws + 512 + 65536 * 4);
    for (int k = 0; k < n_ops; ++k) {
        const SparkChainOp& o = ops[k];
        tc::ChainOp& c = pr.op[k];
        SPARK_REQUIRE(o.dep[0] < k && o.dep[1] < k, SPARK_ERR_INVALID, "spark_linear_chain: op %d depends on a later op", k);
        c.kind = o.kind;
        c.dep0 = o.dep[0];
        c.dep1 = o.dep[1];
        c.y = o.y;
        if (o.kind == SPARK_CHAIN_SILU_MUL) {
            SPARK_REQUIRE(o.x && o.x2 && o.y && o.ic > 0 && o.dep[0] >= 0 && o.dep[1] >= 0, SPARK_ERR_INVALID,
                          "spark_linear_chain: op %d: SiLU needs gate, up, out, width and both producing ops", k);
            c.g = o.x;
            c.u = o.x2;
            c.n = M * o.ic;
            c.target = grid * (tc::kDecThreads / 32);
            continue;
        }
        SPARK_REQUIRE(o.kind == SPARK_CHAIN_LINEAR, SPARK_ERR_INVALID, "spark_linear_chain: op %d: bad kind", k);
        SPARK_REQUIRE(o.fmt != SPARK_FMT_TWOFOUR && tc_linear_ok(o.fmt, o.wq, o.scales, o.x, SPARK_DTYPE_BF16, o.ic, o.ldx) &&
                          o.y && o.oc > 0,
                      SPARK_ERR_UNSUPPORTED,
                      "spark_linear_chain: op %d: SPFP2/FP3/NVFP4 reference layout, bf16 x, ic %% 256, "
                      "16-byte aligned buffers, ldx %% 8", k);
        const int code_bytes = o.fmt == SPARK_FMT_SPFP2 ? 80 : (o.fmt == SPARK_FMT_FP3 ? 96 : 128);
        const uint64_t row_code = (uint64_t)(o.ic / tc::kUnitCols * code_bytes);
        rc = tc::encode_2d(&pr.wmap[k], CU_TENSOR_MAP_DATA_TYPE_UINT8, o.wq, row_code, (uint64_t)o.oc, row_code,
                           (uint32_t)code_bytes, tc::kRows,
                           o.fmt == SPARK_FMT_NVFP4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        if (o.fmt == SPARK_FMT_SPFP2) {
            pr.smap[k] = pr.wmap[k];
        } else {
            rc = tc::encode_2d(&pr.smap[k], CU_TENSOR_MAP_DATA_TYPE_UINT8, o.scales, (uint64_t)(o.ic / 16),
                               (uint64_t)o.oc, (uint64_t)(o.ic / 16), 16, tc::kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc) return rc;
        }
        rc = tc::encode_2d(&pr.xmap[k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, o.x, (uint64_t)o.ic, (uint64_t)M,
                           (uint64_t)o.ldx * 2, 64, tc::kCN, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        c.fmt = o.fmt;
        c.n_rb = (int)((o.oc + tc::kRows - 1) / tc::kRows);
        c.n_kc = (int)(o.ic / tc::kUnitCols);
        c.units = c.n_rb * c.n_kc;
        c.stage_bytes = tc::kRows * (code_bytes + (o.fmt == SPARK_FMT_SPFP2 ? 0 : 16));
        c.oc = o.oc;
        c.ldy = o.ldy;
        c.bias = o.bias;
        c.bias_dtype = o.bias_dtype;
        c.y_dtype = o.y_dtype;
        c.target = grid * 4;
        SPARK_REQUIRE(counter_next + 4 * c.n_rb <= 65536, SPARK_ERR_UNSUPPORTED, "spark_linear_chain: too many rows");
        c.counters = counters + counter_next;
        counter_next += 4 * c.n_rb;
        c.partials = partials + (int64_t)k * 2 * grid * tc::kCN * tc::kRows;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    {
        static bool done[64] = {};
        if (dev >= 0 && dev < 64 && !done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(tc::k_tc_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kCAlloc);
            if (e != cudaSuccess) return set_error((int)e, "k_tc_chain attribute: %s", cudaGetErrorString(e));
            done[dev] = true;
        }
    }
    // done counters start at zero for every launch
    cudaError_t e = cudaMemsetAsync(pr.done, 0, tc::kMaxOps * sizeof(int), s);
    if (e != cudaSuccess) return set_error((int)e, "spark_linear_chain: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::kCAlloc;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, tc::k_tc_chain, pr);
    if (e != cudaSuccess) return set_error((int)e, "k_tc_chain launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

}  // extern "C"
