// stream.cu -- persistent decode GEMV over a batch of packed linears
// (M <= 16 tokens, bf16 activations, fragment-major "tiled" weights).
//
// y_k[M, oc_k] = x_k[M, ic_k] . decode(W_k)^T (+ bias_k) for every op k of a
// batch, in ONE launch of one CTA per SM.  The work is HBM-bound at decode
// batch sizes, so the design keeps every warp streaming weights from its
// first unit to its last:
//   * the batch's units (16 rows x 256 columns of one op) form one sequence,
//     op after op, row group after row group, column chunk fastest; it is cut
//     into G * kCW equal contiguous ranges, one per warp of the grid, so a warp
//     sums whole row groups in registers and shares a row group with another
//     warp only at the two ends of its range;
//   * each warp feeds itself: lane 0 keeps kDepth bulk copies (evict-first in
//     L2) of the warp's next units in flight into the warp's own shared-memory
//     slots, so no warp ever waits for another one's progress;
//   * the warp decodes a staged unit in registers and feeds mma.sync (bf16,
//     fp32 accumulation); a row group shared between warps is summed
//     deterministically (partials + counter; the warp whose range ends in
//     the row group adds them in unit order);
//   * an op that reads an earlier op's output starts a new segment of the
//     sequence (cut the same way): before it reads such an input a warp waits
//     (bounded) until every warp has finished the producing segment, while its
//     weights are already in flight.
//
// Every decoded weight is exact in bf16 (SPFP2 values are powers of two,
// block_fp2_emu.py:36; FP3 / e2m1 codes have <= 2 significant bits and e4m3
// scales <= 4, fp3_emu.py:47, nvfp4_emu.py:109-123), so mma.m16n8k16.bf16
// reads the caller's bf16 x directly.
//
// The main path runs every format on the f16 MMA: the decoded weights are
// exact in f16 too (SPFP2: exponent field e + 5; FP3 / NVFP4 code values
// times an e4m3 scale have at most 6 significant bits and lie within
// [2^-10, 2688]), and f16 has single-instruction conversions from e5m2 and
// e2m1 pairs: SPFP2 becomes e5m2 bytes by one byte permute per four weights,
// FP3 (repacked at tile time) and NVFP4 are e2m1 codes.  The activations are
// converted once per launch, per 256-column chunk and token, to f16 times a
// power of two sigma (max |x| * sigma in [2^14, 2^15), so the conversion of a
// bf16 value is exact down to max |x| * 2^-28); a unit's fresh accumulators
// are scaled by 1 / sigma into the row sums.  The first warp to need a chunk
// claims it (flag 0 -> 1), converts it and publishes it (2; 3 when it holds an
// inf or NaN: the op then runs on the bf16 path, which keeps the
// reference's inf / NaN pattern).
#include <algorithm>
#include <mutex>
#include <new>

#include "common.cuh"

namespace spark {
namespace stream {

constexpr int kCW = 16;                       // warps of a CTA; each streams its own units
constexpr int kThreads = kCW * 32;            // 128 registers a thread
constexpr int kDepth = 6;                     // units in flight per warp
constexpr int kSlotBytes = 2304;              // largest tiled unit (NVFP4)
constexpr int kWarpRing = kDepth * kSlotBytes;
constexpr int kMaxOps = 48;
constexpr int kMaxTok = 16;
constexpr size_t kPartAreaBudget = (size_t)16 << 20;   // partial-sum areas of a batch: one per segment up to this
constexpr uint64_t kWaitNs = 2000000000ull;   // bounded waits: 2 s

// Control block inside the caller's workspace (bytes; the error word is at 0).
constexpr size_t kCtlAbort = 4;
constexpr size_t kCtlCtaDone = 8;
constexpr size_t kCtlSegDone = 64;            // int[kMaxOps]: warps done with each segment
static_assert(kCtlSegDone + 4 * kMaxOps <= 4096, "control block overflows its 4 KB");

struct Op {
    const uint8_t* w;        // tiled weight
    const uint16_t* x;       // bf16 [M][ldx]
    void* y;
    const void* bias;
    int64_t ldx, ldy;
    int fmt, oc, n_kc, ub;   // ub: the op's first unit in the batch's sequence
    int units, unit_bytes, cnt_off, seg;
    int dseg0, dseg1, y_dtype, bias_dtype;   // dseg: segments whose completion the op's input needs (-1: none)
    int silu, f16, flag_off, chunk0;  // f16: the f16 path; flag_off: the op's chunk flags in the counters
                                      // (kFlagStride ints apart);
                                      // chunk0: its first chunk in the batch's converted-activation arrays
    int feed, feed_rgs, feed_cnt, fed;   // feed: 1 + the op whose activation chunks this op's rows complete
                                         // (0: none), feed_rgs row groups per chunk, counters at feed_cnt
                                         // (kFlagStride apart); fed: 1 + that producer (on the consumer)
};

// A segment: ops k0..k1-1, units [ub, ub + units) of the sequence, split over
// T = G * kCW warps: warp v holds q + (v < rem) units from ub + v * q + min(v, rem).
constexpr int kFlagStride = 32;       // ints between two chunk flags (one 128-byte line each)
constexpr int kF16Units = 40;         // below this many units per warp, an all-SPFP2 batch keeps the bf16 path

struct Seg {
    int ub, units, q, rem;
    int k0, k1, active, waited;   // active: warps with a non-empty range; waited: something waits for it
};

struct Args {
    Op op[kMaxOps];
    Seg seg[kMaxOps];
    int n_ops, n_seg, M, n_cnt;
    int part_ring, n_cnt_all;  // part_ring: partial-sum areas, reused every part_ring segments;
                               // n_cnt_all: counters including the chunk flags (reset at the end)
    int n_chunks, pad1;        // chunks of the f16 ops' converted activations
    uint8_t* ws;
    int* counters;
    float* partials;
    int64_t part_stride;     // floats per area: T * 2 * M * 16
    float* xinv;             // [chunk][16]: 1 / sigma per token
    uint16_t* xh;            // [chunk][M][256]: f16 activations times sigma
    // the fused all-reduce of one op (ar_world = 0: none): every rank's
    // receive buffer [2][world][ar_nrg][M][16] of tagged words, as this
    // process maps them, and this rank's call counter
    uint64_t* ar_recv[SPARK_MAX_PEERS];
    int* ar_counter;
    int ar_world, ar_rank, ar_nrg, ar_op;
    float* ar_local;         // the op's rank-local sums [M][ar_nrg * 16] (the op's y during the launch)
    void* ar_y;              // the op's real output, bias and dtypes
    const void* ar_bias;
    int64_t ar_ldy;
    int ar_oc, ar_y_dtype, ar_bias_dtype, pad2;
};

constexpr size_t kXhBudget = (size_t)8 << 20;   // converted activations of a batch's f16 ops

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A . B (+ C) on f16 operands, fp32 accumulation
template <bool ACC>
__device__ __forceinline__ void mma_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    if constexpr (ACC)
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%10,%10,%10};"
            : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// the four e5m2 bytes of v as f16 pairs (bytes 0, 1) and (2, 3); exact
__device__ __forceinline__ void e5m2x4_f16(uint32_t v, uint32_t& lo, uint32_t& hi) {
    asm("{ .reg .b16 l, h; mov.b32 {l, h}, %2; cvt.rn.f16x2.e5m2x2 %0, l; cvt.rn.f16x2.e5m2x2 %1, h; }"
        : "=r"(lo), "=r"(hi)
        : "r"(v));
}
// the eight e2m1 codes of v (code 2j + i in byte j, i = 0 the low nibble) as
// f16 pairs d[j] = (code 2j, code 2j + 1); exact
__device__ __forceinline__ void e2m1x8_f16(uint32_t v, uint32_t* d) {
    asm("{ .reg .b8 b0, b1, b2, b3; mov.b32 {b0, b1, b2, b3}, %4; cvt.rn.f16x2.e2m1x2 %0, b0; "
        "cvt.rn.f16x2.e2m1x2 %1, b1; cvt.rn.f16x2.e2m1x2 %2, b2; cvt.rn.f16x2.e2m1x2 %3, b3; }"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(v));
}
// byte k of w (an e4m3 scale) as an f16 pair (s, s); exact
__device__ __forceinline__ uint32_t e4m3_f16_dup(uint32_t w, int k) {
    const uint32_t b = prmt(w, 0u, 0x4400u | (uint32_t)(k * 0x11));
    uint32_t d;
    asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; cvt.rn.f16x2.e4m3x2 %0, l; }" : "=r"(d) : "r"(b));
    return d;
}
// FP3 step j (0..3) of a tiled code-word group w[0..2]: the eight codes as
// e2m1 nibbles (see fp3_pack_tiled in gemv.cu)
__device__ __forceinline__ uint32_t fp3_e2m1(const uint32_t* w, int j) {
    if (j < 3) return w[j] & 0xbbbbbbbbu;
    return ((w[0] >> 2) & 0x11111111u) | ((w[1] >> 1) & 0x22222222u) | ((w[2] << 1) & 0x88888888u);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// activations that no op of the batch writes: read-only path; those that an
// earlier op of the batch produced: L2 (coherent within the launch)
template <bool PROD>
__device__ __forceinline__ uint4 ld_x(const void* p) {
    uint4 v;
    if constexpr (PROD)
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    else
        asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// activations this launch converted (read after an acquire of their flag)
__device__ __forceinline__ uint4 ld_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Bounded wait on a shared-memory barrier phase.  False (and the abort flags
// raised) once kWaitNs pass, or when another warp has raised an abort flag.
// Bounded wait for a ring slot.  The global abort word and the clock are
// read every 16th round only: thousands of warps reading one global word in
// a tight loop make its L2 line a hot spot in the middle of the weight stream.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* s_abort, volatile int* g_abort,
                                           int* err) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t dl = globaltimer_ns() + kWaitNs;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (*s_abort) return false;
        if ((i & 15u) == 0) {
            if (*g_abort) return false;
            if (globaltimer_ns() > dl) {
                report_device_error(err, 1);
                *s_abort = 1;
                *g_abort = 1;
                return false;
            }
        }
    }
}

// Bounded wait (one thread) until a device counter reaches `target`.
__device__ __forceinline__ bool wait_count(const int* p, int target, volatile int* abort, int* err) {
    if (ld_acquire(p) >= target) return true;
    const uint64_t dl = globaltimer_ns() + kWaitNs;
    unsigned ns = 64;
    while (true) {
        __nanosleep(ns);
        ns = min(2 * ns, 1024u);
        if (ld_acquire(p) >= target) return true;
        if (*abort) return false;
        if (globaltimer_ns() > dl) {
            report_device_error(err, 1);
            *abort = 1;
            return false;
        }
    }
}

// ---------------------------------------------------------------- work split
// Sub-ranges are empty only when q == 0, and then only for v >= rem: the
// warps that share a row group are a contiguous range of v.
__device__ __forceinline__ int vw_start(const Seg& sg, int v) { return v * sg.q + min(v, sg.rem); }
__device__ __forceinline__ int vw_owner(const Seg& sg, int u) {
    const int big = sg.rem * (sg.q + 1);
    return u < big ? u / (sg.q + 1) : sg.rem + (u - big) / sg.q;
}

// The first segment s' >= s in which warp v has units: its range [gu, gend)
// (positions in the batch's sequence).  False when there is none.
__device__ __forceinline__ bool find_range(const Args& a, int v, int& s, int& gu, int& gend) {
    for (; s < a.n_seg; ++s) {
        const Seg& sg = a.seg[s];
        const int n = sg.q + (v < sg.rem ? 1 : 0);
        if (n > 0) {
            gu = sg.ub + vw_start(sg, v);
            gend = gu + n;
            return true;
        }
    }
    return false;
}

// ---------------------------------------------------------------- decoders
// 32-bit window of a little-endian word array starting at bit `pos`.
template <int N>
__device__ __forceinline__ uint32_t window(const uint32_t* c, int pos) {
    const int w = pos >> 5, s = pos & 31;
    if (s == 0) return c[w];
    const uint32_t hi = (w + 1 < N) ? c[w + 1] : 0u;
    return __funnelshift_r(c[w], hi, s);
}

// bf16 bits of an FP3 (3-bit) or e2m1 (4-bit) code (fp3_emu.py:47, nvfp4_emu.py:109-123)
__device__ __forceinline__ uint32_t code_bf16(int fmt, uint32_t code) {
    const int bits = fmt == SPARK_FMT_FP3 ? 3 : 4;
    const uint32_t mag = code & ((1u << (bits - 1)) - 1u), neg = code >> (bits - 1);
    const float tab[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    return (__float_as_uint(tab[mag]) >> 16) | (neg << 15);
}

// FP3 / NVFP4, step s (8 columns) of one row's chunk: four bf16x2 A registers,
// the natural column pairs (2j, 2j + 1), each a table value times the block's
// e4m3 scale (exact in bf16).  Both formats decode e2m1 codes (FP3's tiled
// words become e2m1 nibbles), pair_tab[b] = the two codes of byte b.
template <int FMT>
__device__ __forceinline__ void decode_scaled(const uint32_t* c, uint32_t scale_word, int s, const uint32_t* pair_tab,
                                              const uint32_t* scale_tab, uint32_t* A) {
    const uint32_t s2 = scale_tab[(scale_word >> (8 * (s >> 1))) & 0xffu];
    const uint32_t v = FMT == SPARK_FMT_FP3 ? fp3_e2m1(c + 3 * (s >> 2), s & 3) : c[s];
#pragma unroll
    for (int j = 0; j < 4; ++j) A[j] = bmul2(pair_tab[(v >> (8 * j)) & 0xffu], s2);
}

// SPFP2, block s of rows g and g + 8 from the block's code word W: bf16 pairs
// of columns (2j, 2j + 1).  TL = [L, L, 0, 0] and TH = [H, H | 0x80, 0, 0]
// are the byte tables of a row's block exponent (bf16 of +-2^(e-10) has
// biased exponent E = 117 + e: high byte sign | E >> 1, low byte
// (E & 1) << 7); code c selects byte c of TL and byte c of TH (codes 2 and 3
// are zero).  y = (W >> 2j) & 0x03030303 holds the codes (a, b, c, d) of
// columns 2j, 2j + 1 of row g, then of row g + 8, one a byte; y * 0x11 +
// 0x4040 is the byte-permute selector (a, 4 + a, b, 4 + b) of row g, the
// high word of y * 0x110000, + 0x4040, the one of row g + 8.
__device__ __forceinline__ void decode_spfp2_bf16(uint32_t W, uint32_t TLg, uint32_t THg, uint32_t TLh, uint32_t THh,
                                                  uint32_t* A0, uint32_t* A1) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t y = (W >> (2 * j)) & 0x03030303u;
        A0[j] = prmt(TLg, THg, y * 0x11u + 0x4040u);
        A1[j] = prmt(TLh, THh, __umulhi(y, 0x110000u) + 0x4040u);
    }
}

// Words of this thread's fragment from a staged unit (lane-interleaved
// 16-byte vectors, then an 8-byte tail).
template <int FW>
__device__ __forceinline__ void load_frag(const uint8_t* slot, int lane, uint32_t* fw) {
    constexpr int NV = FW / 4;
    const uint4* v = reinterpret_cast<const uint4*>(slot);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const uint4 q = v[i * 32 + lane];
        fw[4 * i] = q.x;
        fw[4 * i + 1] = q.y;
        fw[4 * i + 2] = q.z;
        fw[4 * i + 3] = q.w;
    }
    const uint2 q = reinterpret_cast<const uint2*>(slot + NV * 512)[lane];
    fw[4 * NV] = q.x;
    fw[4 * NV + 1] = q.y;
}

// One unit of any format: 8 steps of 8 columns, rows g and g + 8, NTB token
// tiles of 8; acc[0] / acc[1] take the two MMAs of a step.  xr[j]: the row of
// x this lane feeds to token tile j (lanes past the last token repeat it; the
// columns they produce are never written).
template <int FMT, int NTB, bool PROD>
__device__ __forceinline__ void unit_mma(const uint32_t* fw, const uint16_t* const (&xr)[NTB], int64_t col,
                                         const uint32_t* pair_tab, const uint32_t* scale_tab,
                                         float (&acc)[2][NTB][4], uint32_t xl) {
    // one token tile: the unit's activations for all 8 steps are loaded first,
    // so their latency overlaps the decode.  Only lanes that feed a real
    // token load (bit 0 of xl); the others feed zeros, to columns that are
    // never written, and keep the L1 return path free.  (Two token tiles load
    // step by step, every lane: predicating those loads measured slower.)
    uint4 xs[NTB == 1 ? 8 : 1];
    if constexpr (NTB == 1) {
#pragma unroll
        for (int s = 0; s < 8; ++s) xs[s] = (xl & 1u) ? ld_x<PROD>(xr[0] + col + 8 * s) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t A0[4], A1[4];
        if constexpr (FMT == SPARK_FMT_SPFP2) {
            // exponent byte tables of four blocks at once, rows g (low
            // nibbles) and g + 8 (high nibbles): bytes 117 + e, then H and L
            const uint32_t E = fw[8 + (s >> 2)];
            const uint32_t Yg = (E & 0x0f0f0f0fu) + 0x75757575u, Yh = ((E >> 4) & 0x0f0f0f0fu) + 0x75757575u;
            const uint32_t Hg = (Yg >> 1) & 0x7f7f7f7fu, Lg = (Yg << 7) & 0x80808080u;
            const uint32_t Hh = (Yh >> 1) & 0x7f7f7f7fu, Lh = (Yh << 7) & 0x80808080u;
            const uint32_t k = (uint32_t)(s & 3);
            const uint32_t selH = 0x8800u | ((4u + k) << 4) | k, selL = 0x4400u | (k << 4) | k;
            decode_spfp2_bf16(fw[s], prmt(Lg, 0u, selL), prmt(Hg, Hg | 0x80808080u, selH), prmt(Lh, 0u, selL),
                              prmt(Hh, Hh | 0x80808080u, selH), A0, A1);
        } else {
            constexpr int CW = FMT == SPARK_FMT_FP3 ? 6 : 8;
            decode_scaled<FMT>(fw, fw[CW], s, pair_tab, scale_tab, A0);
            decode_scaled<FMT>(fw + CW + 1, fw[2 * CW + 1], s, pair_tab, scale_tab, A1);
        }
#pragma unroll
        for (int j = 0; j < NTB; ++j) {
            uint4 x;
            if constexpr (NTB == 1) x = xs[s];
            else x = ld_x<PROD>(xr[j] + col + 8 * s);
            mma_bf16(acc[0][j], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
            mma_bf16(acc[1][j], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
        }
    }
}

// f16 path, step s of rows g (A0) and g + 8 (A1): four f16 pairs each.
// SPFP2: the e5m2 bytes of columns (0, 4, 1, 5) and (2, 6, 3, 7) (nibbles of
// W & 0x3333 and W >> 2 & 0x3333; row g + 8 from W >> 16), T = [B, B | 0x80,
// 0, 0] with B = (e + 5) << 2 the block's byte table; pairs (0, 4) (1, 5)
// (2, 6) (3, 7), the order the activations are converted in.  FP3 / NVFP4:
// e2m1 pairs (2j, 2j + 1) times the block's scale.
template <int FMT>
__device__ __forceinline__ void decode_f16(const uint32_t* fw, int s, uint32_t* A0, uint32_t* A1) {
    if constexpr (FMT == SPARK_FMT_SPFP2) {
        const uint32_t E = fw[8 + (s >> 2)];
        const uint32_t Bg = (E & 0x0f0f0f0fu) * 4u + 0x14141414u, Bh = ((E >> 4) & 0x0f0f0f0fu) * 4u + 0x14141414u;
        const uint32_t k = (uint32_t)(s & 3);
        const uint32_t sel = 0x8800u | ((4u + k) << 4) | k;
        const uint32_t Tg = prmt(Bg, Bg | 0x80808080u, sel), Th = prmt(Bh, Bh | 0x80808080u, sel);
        const uint32_t W = fw[s];
        e5m2x4_f16(prmt(Tg, 0u, W & 0x3333u), A0[0], A0[1]);
        e5m2x4_f16(prmt(Tg, 0u, (W >> 2) & 0x3333u), A0[2], A0[3]);
        e5m2x4_f16(prmt(Th, 0u, (W >> 16) & 0x3333u), A1[0], A1[1]);
        e5m2x4_f16(prmt(Th, 0u, (W >> 18) & 0x3333u), A1[2], A1[3]);
    } else {
        constexpr int CW = FMT == SPARK_FMT_FP3 ? 6 : 8;
        const uint32_t vg = FMT == SPARK_FMT_FP3 ? fp3_e2m1(fw + 3 * (s >> 2), s & 3) : fw[s];
        const uint32_t vh = FMT == SPARK_FMT_FP3 ? fp3_e2m1(fw + CW + 1 + 3 * (s >> 2), s & 3) : fw[CW + 1 + s];
        const uint32_t sg = e4m3_f16_dup(fw[CW], s >> 1), sh = e4m3_f16_dup(fw[2 * CW + 1], s >> 1);
        e2m1x8_f16(vg, A0);
        e2m1x8_f16(vh, A1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            A0[j] = hmul2(A0[j], sg);
            A1[j] = hmul2(A1[j], sh);
        }
    }
}

// f16 path, one unit into fresh accumulators.  xr[j]: this lane's row of the
// converted activations for token tile j, at the unit's chunk.
template <int FMT, int NTB>
__device__ __forceinline__ void unit_h(const uint32_t* fw, const uint16_t* const (&xr)[NTB], float (&acc)[2][NTB][4]) {
    uint4 xs[NTB == 1 ? 8 : 1];
    if constexpr (NTB == 1) {
#pragma unroll
        for (int s = 0; s < 8; ++s) xs[s] = ld_v4(xr[0] + 8 * s);
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t A0[4], A1[4];
        decode_f16<FMT>(fw, s, A0, A1);
#pragma unroll
        for (int j = 0; j < NTB; ++j) {
            uint4 x;
            if constexpr (NTB == 1) x = xs[s];
            else x = ld_v4(xr[j] + 8 * s);
            if (s == 0) {
                mma_f16<false>(acc[0][j], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
                mma_f16<false>(acc[1][j], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
            } else {
                mma_f16<true>(acc[0][j], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
                mma_f16<true>(acc[1][j], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
            }
        }
    }
}

// f16 path, one token tile: xs holds this unit's activations (loaded during
// the unit before); each step's register is refilled with the next unit's
// (nxt, when the op has one) as soon as its MMAs have read it, so the loads
// overlap a whole unit of decoding.
template <int FMT>
__device__ __forceinline__ void unit_h1(const uint32_t* fw, uint4 (&xs)[8], const uint16_t* nxt,
                                        float (&acc)[2][1][4]) {
    // nxt: null after the op's last unit, and for lanes past the last token
    // when there are several tokens (they keep feeding zeros and load nothing)
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t A0[4], A1[4];
        decode_f16<FMT>(fw, s, A0, A1);
        const uint4 x = xs[s];
        if (s == 0) {
            mma_f16<false>(acc[0][0], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
            mma_f16<false>(acc[1][0], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
        } else {
            mma_f16<true>(acc[0][0], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
            mma_f16<true>(acc[1][0], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
        }
        if (nxt) xs[s] = ld_v4(nxt + 8 * s);
    }
}

// ---------------------------------------------------------------- epilogue
__device__ __forceinline__ float bias_at(const Op& op, int64_t row) {
    return op.bias ? load_as_float(op.bias, op.bias_dtype, row) : 0.0f;
}

__device__ __forceinline__ float silu_mul(float gv, float uv) { return gv / (1.0f + __expf(-gv)) * uv; }

struct Ctl {
    int* err;
    volatile int* abort;
    int* seg_done;
};

// ---------------------------------------------------------------- fused all-reduce
// All-reduce of one finished row group over the ranks, in two halves.  Every
// value travels as one 8-byte word: the fp32 bits in the low half, the call
// number in the high half, written and read with single 64-bit accesses (a
// naturally aligned 64-bit access is single-copy atomic, over NVLink too), so
// a reader that sees this call's number sees the value: no release fence,
// no flag round trip.
// ar_publish: this lane's values val[e] (token mm[e], row rr[e] of the group,
// valid ok[e]) into every rank's receive slot for (this rank, rg).
// ar_collect: val[e] becomes the sum over ranks 0..W-1 in that order, each
// term waited for (bounded) until its word carries this call's number (this
// rank's own term from registers: the same bits the others read).  Slots
// alternate by call parity; a rank writes a slot two calls later only after
// it has read every rank's words of the call in between, so every rank has
// finished with that slot.
__device__ __forceinline__ uint32_t ar_epoch(const Args& a) {
    // this call's number: the calls this rank made before it, + 1
    return (uint32_t)*reinterpret_cast<volatile int*>(a.ar_counter) + 1u;
}
__device__ __forceinline__ void st_word_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
template <int NE>
__device__ void ar_publish(const Args& a, int rg, const int (&mm)[NE], const int (&rr)[NE], const float (&val)[NE],
                           const bool (&ok)[NE], uint32_t epoch) {
    const int W = a.ar_world, R = a.ar_rank, nrg = a.ar_nrg, M = a.M;
    const int64_t stride = (int64_t)nrg * M * 16;                             // one rank's slots
    const int64_t off = ((int64_t)(epoch & 1u) * W * nrg + rg) * M * 16;      // (parity, rank 0, rg)
    for (int p = 0; p < W; ++p) {
        uint64_t* dst = a.ar_recv[p] + off + R * stride;
#pragma unroll
        for (int e = 0; e < NE; ++e)
            if (ok[e]) st_word_sys(dst + mm[e] * 16 + rr[e], (uint64_t)epoch << 32 | __float_as_uint(val[e]));
    }
}
template <int NE>
__device__ bool ar_collect(const Args& a, const Ctl& C, int rg, const int (&mm)[NE], const int (&rr)[NE],
                           float (&val)[NE], const bool (&ok)[NE], uint32_t epoch) {
    const int W = a.ar_world, R = a.ar_rank, nrg = a.ar_nrg, M = a.M;
    const int64_t stride = (int64_t)nrg * M * 16;
    const int64_t off = ((int64_t)(epoch & 1u) * W * nrg + rg) * M * 16;
    const uint64_t* base = a.ar_recv[R] + off;
    bool good = true;
#pragma unroll
    for (int e = 0; e < NE; ++e) {
        if (!ok[e]) continue;
        float sum = 0.0f;
        for (int r = 0; r < W; ++r) {
            if (r == R) {
                sum += val[e];
                continue;
            }
            const uint64_t* q = base + r * stride + mm[e] * 16 + rr[e];
            uint64_t w = ld_word_sys(q);
            if ((uint32_t)(w >> 32) != epoch && good) {
                const uint64_t dl = globaltimer_ns() + kWaitNs;
                unsigned ns = 32;
                while ((uint32_t)((w = ld_word_sys(q)) >> 32) != epoch) {
                    if (*C.abort || globaltimer_ns() > dl) {
                        if (!*C.abort) report_device_error(C.err, 5);
                        *C.abort = 1;
                        good = false;
                        break;
                    }
                    __nanosleep(ns);
                    ns = min(2 * ns, 256u);
                }
            }
            sum += __uint_as_float((uint32_t)w);
        }
        val[e] = sum;
    }
    return __all_sync(0xffffffffu, good);
}

// The exchange of the all-reduced op, after this warp's units of it: the op
// itself wrote this rank's sums (fp32, no bias) to the local buffer ar_local
// ([M][ar_nrg * 16]); the row groups r_lo..r_hi are the ones this warp
// finished (their first unit lies in its range).  All are published first,
// then each is summed over the ranks and written to the op's real output.
__device__ __noinline__ void ar_pass(const Args& a, const Ctl& C, int r_lo, int r_hi, int lane) {
    const int M = a.M, ld = a.ar_nrg * 16;
    __syncwarp();                     // this warp's own row writes before its reads
    const int row = lane & 15;
    constexpr int NE = 8;
    const uint32_t epoch = ar_epoch(a);
    for (int pass = 0; pass < 2; ++pass)
        for (int rg = r_lo; rg <= r_hi; ++rg) {
            int mm[NE], rr[NE];
            float val[NE];
            bool ok[NE];
#pragma unroll
            for (int i = 0; i < NE; ++i) {
                mm[i] = (lane >> 4) + 2 * i;
                rr[i] = row;
                ok[i] = mm[i] < M;
                val[i] = ok[i] ? __ldcg(a.ar_local + (int64_t)mm[i] * ld + rg * 16 + row) : 0.0f;
            }
            if (pass == 0) {
                ar_publish<NE>(a, rg, mm, rr, val, ok, epoch);
                continue;
            }
            if (!ar_collect<NE>(a, C, rg, mm, rr, val, ok, epoch)) return;
            const int64_t r = (int64_t)rg * 16 + row;
#pragma unroll
            for (int i = 0; i < NE; ++i) {
                if (!ok[i] || r >= a.ar_oc) continue;
                const float b = a.ar_bias ? load_as_float(a.ar_bias, a.ar_bias_dtype, r) : 0.0f;
                store_from_float(a.ar_y, a.ar_y_dtype, (int64_t)mm[i] * a.ar_ldy + r, val[i] + b);
            }
        }
}

template <bool PROD>
__device__ __noinline__ void prep_chunk(const Args& a, int k, int c, int lane);

// A consumer on the bf16 path (no conversion) that its producer feeds: wait
// (bounded, growing sleeps) until every row group of the chunks that units
// [u0, u1) of op k read is written.
__device__ __noinline__ bool wait_fed(const Args& a, const Ctl& C, int k, int u0, int u1, int lane) {
    const Op& op = a.op[k];
    const Op& pr = a.op[op.fed - 1];
    const int n = op.n_kc, L = min(u1 - u0, n), c0 = u0 % n;
    bool ok = true;
    for (int b0 = 0; b0 < L && ok; b0 += 32) {
        int c = c0 + b0 + lane;
        c -= c >= n ? n : 0;
        c -= c >= n ? n : 0;
        if (b0 + lane < L) {
            const int* cnt = a.counters + pr.feed_cnt + c * kFlagStride;
            if (ld_acquire(cnt) < pr.feed_rgs) {
                const uint64_t dl = globaltimer_ns() + kWaitNs;
                unsigned ns = 64;
                while (ld_acquire(cnt) < pr.feed_rgs) {
                    if (*C.abort) {
                        ok = false;
                        break;
                    }
                    if (globaltimer_ns() > dl) {
                        report_device_error(C.err, 1);
                        *C.abort = 1;
                        ok = false;
                        break;
                    }
                    __nanosleep(ns);
                    ns = min(2 * ns, 1024u);
                }
            }
        }
        ok = __all_sync(0xffffffffu, ok);   // every lane's acquire before any lane's reads
    }
    return ok;
}
// Op k feeds a later op's converted activations.  After its units of op k,
// a warp counts the row groups it wrote (r_lo..r_hi, those whose first unit
// lies in its range) toward their chunks; the warp that completes a chunk
// converts it, so the consumer waits only for the chunks it reads, not for
// the whole producing segment.  (The warp barrier orders every lane's rows
// before lane 0's release; the completing warp's acquire orders the other
// writers' rows before its reads.)
__device__ __noinline__ void feed_pass(const Args& a, int k, int r_lo, int r_hi, int lane) {
    const Op& op = a.op[k];
    __syncwarp();
    for (int c = r_lo / op.feed_rgs; c <= r_hi / op.feed_rgs; ++c) {
        const int n = min(r_hi, (c + 1) * op.feed_rgs - 1) - max(r_lo, c * op.feed_rgs) + 1;
        int* cnt = a.counters + op.feed_cnt + c * kFlagStride;
        int old = 0;
        if (lane == 0) {
            asm volatile("atom.release.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(cnt), "r"(n) : "memory");
            if (old + n == op.feed_rgs) (void)ld_acquire(cnt);
        }
        if (__shfl_sync(0xffffffffu, old, 0) + n == op.feed_rgs && a.op[op.feed - 1].f16)
            prep_chunk<true>(a, op.feed - 1, c, lane);
    }
}

// Row-group values are held as v[2j + i][r] = row g (r = 0) / g + 8 (r = 1)
// of token 8j + 2t + i.  write_rows writes a whole row group; flush_partial
// publishes the partial of a shared one.  The first contributor (the warp
// whose range ends in the row group, or begins at its first unit) sums the
// partials in unit order and writes the rows: it reaches the row group last
// (the others meet it at the start of their ranges), so it rarely waits, and
// the others publish without waiting for a round trip.
template <int NV>
__device__ __forceinline__ void write_rows(const Op& op, int M, int rg, const float (&v)[NV][2], int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int64_t r0 = (int64_t)rg * 16 + g, r1 = r0 + 8;
    const float b0 = r0 < op.oc ? bias_at(op, r0) : 0.0f, b1 = r1 < op.oc ? bias_at(op, r1) : 0.0f;
#pragma unroll
    for (int idx = 0; idx < NV; ++idx) {
        const int m = 8 * (idx >> 1) + 2 * t + (idx & 1);
        if (m >= M) continue;
        if (op.silu) {
            // rows g (gate) and g + 8 (its up row) -> column 8 rg + g
            store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + (int64_t)rg * 8 + g,
                             silu_mul(v[idx][0] + b0, v[idx][1] + b1));
            continue;
        }
        if (r0 < op.oc) store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r0, v[idx][0] + b0);
        if (r1 < op.oc) store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r1, v[idx][1] + b1);
    }
}

// slot: 0 for the row group holding the start of this warp's range in the
// segment, 1 for the one holding its end.
template <int NV>
__device__ __noinline__ void flush_partial(const Args& a, const Ctl& C, int s, int k, int vw, int rg, int slot,
                                           const float (&v)[NV][2], int lane) {
    const Op& op = a.op[k];
    const Seg& sg = a.seg[s];
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M;
    float* area = a.partials + (int64_t)(s % a.part_ring) * a.part_stride;
    // areas are reused every part_ring segments: the segment that last used
    // this one must be finished (every warp past it, its partials read)
    if (s >= a.part_ring) {
        bool ok = true;
        if (lane == 0) ok = wait_count(C.seg_done + (s - a.part_ring), a.seg[s - a.part_ring].active, C.abort, C.err);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
    }
    float* mine = area + ((int64_t)vw * 2 + slot) * M * 16;
#pragma unroll
    for (int idx = 0; idx < NV; ++idx) {
        const int m = 8 * (idx >> 1) + 2 * t + (idx & 1);
        if (m < M) {
            __stcg(mine + m * 16 + g, v[idx][0]);
            __stcg(mine + m * 16 + g + 8, v[idx][1]);
        }
    }
    // the warp barrier orders every lane's partial before lane 0's release.
    // (No GPU-scope fence here: lane 0 has bulk copies in flight, and a fence
    // would wait for them.)
    __syncwarp();
    const int first = op.ub + rg * op.n_kc - sg.ub;        // the row group's units in segment order
    const int v_lo = vw_owner(sg, first), v_hi = vw_owner(sg, first + op.n_kc - 1);
    int* cnt = a.counters + op.cnt_off + rg;
    if (vw != v_lo) {
        if (lane == 0) red_release_add(cnt, 1);
        return;
    }
    // the others never wait on this warp, so the wait ends; bounded all the same
    bool ok = true;
    if (lane == 0) ok = wait_count(cnt, v_hi - v_lo, C.abort, C.err);
    if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;   // lane 0's acquire before every lane's reads
    // the first contributor holds this row group in its second slot when its
    // range began before the row group
    const int lo_slot = vw_start(sg, v_lo) < first ? 1 : 0;
    const int row = lane & 15;
    const int64_t r = (int64_t)rg * 16 + row;
    const float b = op.silu ? (row < 8 ? bias_at(op, r) : 0.0f) : (r < op.oc ? bias_at(op, r) : 0.0f);
    const float bu = op.silu && row < 8 ? bias_at(op, r + 8) : 0.0f;
    // lane l: row l & 15 of tokens (l >> 4) + 2i; partials of a batch of 4
    // contributors are loaded before they are added (in unit order)
    for (int i = 0; 2 * i < M; ++i) {
        const int m = (lane >> 4) + 2 * i;
        float sum = 0.0f;
        if (m < M) {
            for (int w0 = v_lo; w0 <= v_hi; w0 += 4) {
                float p[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int w = w0 + j;
                    p[j] = w <= v_hi ? __ldcg(area + ((int64_t)w * 2 + (w == v_lo ? lo_slot : 0)) * M * 16 + m * 16 + row)
                                     : 0.0f;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) sum += p[j];
            }
        }
        if (op.silu) {
            const float up = __shfl_down_sync(0xffffffffu, sum, 8);
            if (m < M && row < 8)
                store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + (int64_t)rg * 8 + row,
                                 silu_mul(sum + b, up + bu));
        } else if (m < M && r < op.oc) {
            store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r, sum + b);
        }
    }
    if (lane == 0) *cnt = 0;
}

// ---------------------------------------------------------------- converted activations
__device__ __forceinline__ void st_release(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t f16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// Convert chunk c (256 columns) of op k's activations, one warp: lane l
// takes columns 8l..8l+7 (step l & 7 of the 64-column slice l >> 3) of every
// token, in the order the op's decoder pairs them (SPFP2: 0, 4, 1, 5, 2, 6,
// 3, 7; FP3 / NVFP4: natural).  Then publish the chunk.
template <bool PROD>
__device__ __noinline__ void prep_chunk(const Args& a, int k, int c, int lane) {
    const Op& op = a.op[k];
    const int M = a.M;
    const int gc = op.chunk0 + c;
    bool bad = false;
    // the next token's load in flight while one is converted
    uint4 nx = ld_x<PROD>(op.x + (int64_t)c * 256 + 8 * lane);
    for (int m = 0; m < M; ++m) {
        const uint4 v = nx;
        if (m + 1 < M) nx = ld_x<PROD>(op.x + (int64_t)(m + 1) * op.ldx + (int64_t)c * 256 + 8 * lane);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float f[8];
        float mx = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            bad |= !isfinite(f[i]);
            mx = fmaxf(mx, fabsf(f[i]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // sigma = 2^(14 - E) for max |x| = 1.f * 2^E (E clamped below at -112)
        const int e = max((int)((__float_as_uint(mx) >> 23) & 0xffu), 15);
        const float sig = mx > 0.0f ? __uint_as_float((uint32_t)(268 - e) << 23) : 1.0f;
        const float inv = mx > 0.0f ? __uint_as_float((uint32_t)(e - 14) << 23) : 1.0f;
        if (lane == 0) a.xinv[(int64_t)gc * 16 + m] = inv;
        uint4 o;
        if (op.fmt == SPARK_FMT_SPFP2)
            o = make_uint4(f16x2_rn(f[0] * sig, f[4] * sig), f16x2_rn(f[1] * sig, f[5] * sig),
                           f16x2_rn(f[2] * sig, f[6] * sig), f16x2_rn(f[3] * sig, f[7] * sig));
        else
            o = make_uint4(f16x2_rn(f[0] * sig, f[1] * sig), f16x2_rn(f[2] * sig, f[3] * sig),
                           f16x2_rn(f[4] * sig, f[5] * sig), f16x2_rn(f[6] * sig, f[7] * sig));
        *reinterpret_cast<uint4*>(a.xh + ((int64_t)gc * M + m) * 256 + 8 * lane) = o;
    }
    if (lane >= M && lane < 16) a.xinv[(int64_t)gc * 16 + lane] = 1.0f;
    bad = __any_sync(0xffffffffu, bad);   // also orders every lane's stores before lane 0's release
    if (lane == 0) st_release(a.counters + op.flag_off + c * kFlagStride, bad ? 3 : 2);
}

// Make the chunks of op k's converted activations that units [u0, u1) of the
// op read ready: claim and prepare the unclaimed ones, then wait (bounded,
// with a growing sleep) for the rest.  Units are row-group major, chunk
// fastest, so the range reads a run of chunks that may wrap.  Only the
// chunks a warp reads are polled: thousands of warps polling every chunk
// flag of an op turn its cache lines into an L2 hot spot that slows the
// weight stream.  bad: one of them holds an inf or NaN (the warp then takes
// the bf16 path for this op).  False on abort.
template <bool PROD>
__device__ bool ensure_chunks(const Args& a, const Ctl& C, int k, int u0, int u1, int lane, bool& bad) {
    const Op& op = a.op[k];
    int* flags = a.counters + op.flag_off;
    const int n = op.n_kc;
    const int L = min(u1 - u0, n), c0 = u0 % n;
    while (!op.fed) {
        int found = -1;
        for (int b0 = 0; b0 < L && found < 0; b0 += 32) {
            int c = c0 + b0 + lane;
            c -= c >= n ? n : 0;
            c -= c >= n ? n : 0;
            const bool free = b0 + lane < L && ld_acquire(flags + c * kFlagStride) == 0;
            const unsigned m = __ballot_sync(0xffffffffu, free);
            if (m) found = __shfl_sync(0xffffffffu, c, __ffs(m) - 1);
        }
        if (found < 0) break;
        int won = 0;
        if (lane == 0) won = atomicCAS(flags + found * kFlagStride, 0, 1) == 0;
        if (__shfl_sync(0xffffffffu, won, 0)) prep_chunk<PROD>(a, k, found, lane);
    }
    bool any_bad = false, ok = true;
    for (int b0 = 0; b0 < L && ok; b0 += 32) {
        int c = c0 + b0 + lane;
        c -= c >= n ? n : 0;
        c -= c >= n ? n : 0;
        int f = 2;
        if (b0 + lane < L) {
            f = ld_acquire(flags + c * kFlagStride);
            if (f < 2) {
                const uint64_t dl = globaltimer_ns() + kWaitNs;
                unsigned ns = 64;
                while ((f = ld_acquire(flags + c * kFlagStride)) < 2) {
                    if (*C.abort) {
                        ok = false;
                        break;
                    }
                    if (globaltimer_ns() > dl) {
                        report_device_error(C.err, 1);
                        *C.abort = 1;
                        ok = false;
                        break;
                    }
                    __nanosleep(ns);
                    ns = min(2 * ns, 1024u);
                }
            }
        }
        any_bad |= f == 3;
        ok = __all_sync(0xffffffffu, ok);
    }
    bad = __any_sync(0xffffffffu, any_bad);   // every flag's acquire before any lane's reads
    return ok;
}

// ---------------------------------------------------------------- the warp's copy stream
// The warp's next unit to copy: a run of `left` units of op k from address
// src (one op inside range [.., gend) of segment s; run_end: the run's end in
// the sequence).  Warp-uniform; lane 0 issues the copies.
struct Feed {
    const uint8_t* src;
    int left, ubytes;
    int s, run_end, gend, k;
    bool live;
    uint32_t slot;           // next slot to fill
    uint32_t n;              // copies issued
};

// Start the run of op k at sequence position gu.
__device__ __forceinline__ void feed_run(const Args& a, Feed& F, int gu) {
    while (F.k + 1 < a.n_ops && gu >= a.op[F.k + 1].ub) ++F.k;
    const Op& op = a.op[F.k];
    F.ubytes = op.unit_bytes;
    F.src = op.w + (int64_t)(gu - op.ub) * op.unit_bytes;
    F.run_end = min(F.gend, op.ub + op.units);
    F.left = F.run_end - gu;
}

__device__ __forceinline__ void feed_next(const Args& a, Feed& F, int vw) {
    int gu = F.run_end;
    if (gu == F.gend) {
        ++F.s;
        F.live = find_range(a, vw, F.s, gu, F.gend);
        if (!F.live) return;
    }
    feed_run(a, F, gu);
}

__device__ __forceinline__ void feed_issue(const Args& a, Feed& F, int vw, uint32_t ring, uint32_t bars, int lane,
                                           uint64_t policy) {
    if (lane == 0) {
        const uint32_t fb = bars + 8 * F.slot;
        mbar_expect_tx(fb, (uint32_t)F.ubytes);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
            "%4;" ::"r"(ring + F.slot * kSlotBytes),
            "l"(F.src), "r"(F.ubytes), "r"(fb), "l"(policy)
            : "memory");
    }
    F.src += F.ubytes;
    F.slot = F.slot + 1 == kDepth ? 0 : F.slot + 1;
    ++F.n;
    if (--F.left == 0) feed_next(a, F, vw);
}

// The consumer side of the same sequence.
struct Walk {
    uint32_t slot, parity;   // next slot to read and its phase parity
    uint32_t n;              // units read
    bool dead;
};

// Process units [gu, end) of op k (all inside one range of segment s, which
// ends at gend).  seg0: the first unit of the row group's part being summed.
template <int FMT, int NTB, bool PROD, bool H = false>
__device__ __forceinline__ void run_units(const Args& a, const Ctl& C, Feed& F, Walk& Wk, int s, int k, int gu,
                                          int end, int gend, int vw, int k_first, int rg_first, const uint8_t* ring_p,
                                          uint32_t ring, uint32_t bars, volatile int* s_abort, const uint32_t* pair_tab,
                                          const uint32_t* scale_tab, int lane, uint64_t policy) {
    const Op& op = a.op[k];
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M;
    const int n_kc = op.n_kc;
    // x rows this lane feeds (token 8j + g; lanes past the last token repeat
    // it): the caller's bf16 rows, or on the f16 path the converted chunks
    const uint16_t* xr[NTB];
    const float* xi = nullptr;          // f16 path: 1 / sigma of tokens 2t, 2t + 1 (+ 8j) per chunk
    int64_t kc_stride = 256;            // elements from one chunk to the next in xr
#pragma unroll
    for (int j = 0; j < NTB; ++j) {
        const int m = min(8 * j + g, M - 1);
        if constexpr (H) xr[j] = a.xh + ((int64_t)op.chunk0 * M + m) * 256 + t * 64;
        else xr[j] = op.x + (int64_t)m * op.ldx + t * 64;
    }
    if constexpr (H) {
        xi = a.xinv + (int64_t)op.chunk0 * 16 + 2 * t;
        kc_stride = 256 * M;
    }
    const uint32_t xl = (g < M ? 1u : 0u) | (8 + g < M ? 2u : 0u);   // token tiles this lane feeds a real token
    // f16 path: with one token every lane loads it (a warp-uniform branch
    // measured faster); with several, lanes past the last token skip the loads
    const bool ldx = M == 1 || (xl & 1u) != 0;
    const int lu0 = gu - op.ub;
    int rg = lu0 / n_kc, kc = lu0 - rg * n_kc;
    int seg0 = gu;
    float acc[2][NTB][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < NTB; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[h][j][i] = 0.0f;
    constexpr int FW = FMT == SPARK_FMT_SPFP2 ? 10 : (FMT == SPARK_FMT_FP3 ? 14 : 18);
    // f16 path, one token tile: the first unit's activations and scales
    uint4 xs[H && NTB == 1 ? 8 : 1];
    float2 rr = make_float2(0.0f, 0.0f);
    if constexpr (H && NTB == 1) {
        const uint16_t* x0 = xr[0] + (int64_t)kc * kc_stride;
#pragma unroll
        for (int q = 0; q < 8; ++q) xs[q] = ldx ? ld_v4(x0 + 8 * q) : make_uint4(0u, 0u, 0u, 0u);
        rr = *reinterpret_cast<const float2*>(xi + kc * 16);
    }
    for (; gu < end; ++gu) {
        const bool ok = __all_sync(0xffffffffu, wait_phase(bars + 8 * Wk.slot, Wk.parity, s_abort, C.abort, C.err));
        if (!ok) {
            Wk.dead = true;
            return;
        }
        uint32_t fw[FW];
        load_frag<FW>(ring_p + Wk.slot * kSlotBytes, lane, fw);
        __syncwarp();
        // the slot's bytes are in registers: refill it with the unit kDepth ahead
        if (F.live) {
            if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            feed_issue(a, F, vw, ring, bars, lane, policy);
        }
        ++Wk.n;
        if (++Wk.slot == kDepth) {
            Wk.slot = 0;
            Wk.parity ^= 1u;
        }

        if constexpr (H && NTB == 1) {
            const bool more = gu + 1 < end;
            const int kn = kc + 1 == n_kc ? 0 : kc + 1;
            float u[2][1][4];
            unit_h1<FMT>(fw, xs, more && ldx ? xr[0] + (int64_t)kn * kc_stride : nullptr, u);
            const float2 r = rr;
            if (more) rr = *reinterpret_cast<const float2*>(xi + kn * 16);
            acc[0][0][0] += (u[0][0][0] + u[1][0][0]) * r.x;
            acc[0][0][1] += (u[0][0][1] + u[1][0][1]) * r.y;
            acc[0][0][2] += (u[0][0][2] + u[1][0][2]) * r.x;
            acc[0][0][3] += (u[0][0][3] + u[1][0][3]) * r.y;
        } else if constexpr (H) {
            const uint16_t* xq[NTB];
#pragma unroll
            for (int j = 0; j < NTB; ++j) xq[j] = xr[j] + (int64_t)kc * kc_stride;
            float u[2][NTB][4];
            unit_h<FMT, NTB>(fw, xq, u);
#pragma unroll
            for (int j = 0; j < NTB; ++j) {
                const float2 r = *reinterpret_cast<const float2*>(xi + kc * 16 + 8 * j);
                acc[0][j][0] += (u[0][j][0] + u[1][j][0]) * r.x;
                acc[0][j][1] += (u[0][j][1] + u[1][j][1]) * r.y;
                acc[0][j][2] += (u[0][j][2] + u[1][j][2]) * r.x;
                acc[0][j][3] += (u[0][j][3] + u[1][j][3]) * r.y;
            }
        } else {
            const uint16_t* xq[NTB];
#pragma unroll
            for (int j = 0; j < NTB; ++j) xq[j] = xr[j];
            unit_mma<FMT, NTB, PROD>(fw, xq, (int64_t)kc * 256, pair_tab, scale_tab, acc, xl);
        }

        if (kc == n_kc - 1 || gu + 1 == gend) {
            float vals[2 * NTB][2];
#pragma unroll
            for (int j = 0; j < NTB; ++j)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    vals[2 * j + i][0] = acc[0][j][i] + acc[1][j][i];
                    vals[2 * j + i][1] = acc[0][j][2 + i] + acc[1][j][2 + i];
                }
            // an all-reduced op's row groups all go through flush_partial (a warp
            // that holds a whole row group is its own finisher there)
            if (kc == n_kc - 1 && seg0 == op.ub + rg * n_kc)
                write_rows<2 * NTB>(op, M, rg, vals, lane);
            else
                flush_partial<2 * NTB>(a, C, s, k, vw, rg, (k == k_first && rg == rg_first) ? 0 : 1, vals, lane);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < NTB; ++j)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[h][j][i] = 0.0f;
            seg0 = gu + 1;
        }
        if (++kc == n_kc) {
            kc = 0;
            ++rg;
        }
    }
}

template <int NTB, bool PROD, bool H>
__device__ __forceinline__ void run_op(const Args& a, const Ctl& C, Feed& F, Walk& Wk, int s, int k, int gu, int end,
                                       int gend, int vw, int k_first, int rg_first, const uint8_t* ring_p, uint32_t ring,
                                       uint32_t bars, volatile int* s_abort, const uint32_t* pair_nv,
                                       const uint32_t* scale_tab, int lane, uint64_t policy) {
    const int fmt = a.op[k].fmt;
    if (fmt == SPARK_FMT_SPFP2)
        run_units<SPARK_FMT_SPFP2, NTB, PROD, H>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring,
                                                 bars, s_abort, pair_nv, scale_tab, lane, policy);
    else if (fmt == SPARK_FMT_FP3)
        run_units<SPARK_FMT_FP3, NTB, PROD, H>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring,
                                               bars, s_abort, pair_nv, scale_tab, lane, policy);
    else
        run_units<SPARK_FMT_NVFP4, NTB, PROD, H>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring,
                                                 bars, s_abort, pair_nv, scale_tab, lane, policy);
}

template <int NTB>
__device__ void warp_main(const Args& a, const Ctl& C, const uint8_t* ring_p, uint32_t ring, uint32_t bars,
                          volatile int* s_abort, const uint32_t* pair_nv, const uint32_t* scale_tab, int vw, int lane) {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    Feed F;
    F.s = 0;
    F.k = 0;
    F.slot = 0;
    F.n = 0;
    {
        int gu = 0;
        F.live = find_range(a, vw, F.s, gu, F.gend);
        if (F.live) feed_run(a, F, gu);
    }
    const bool has_units = F.live;     // (priming clears F.live when the range fits in the ring)
    // prime the ring.  Weights only: with a programmatic launch this runs
    // while the previous kernel of the stream may still be finishing, and no
    // kernel that triggers this launch early writes weights.
    for (int i = 0; i < kDepth && F.live; ++i) feed_issue(a, F, vw, ring, bars, lane, policy);
    // activations, the workspace and the outputs only after the previous grid
    // (a no-op without a programmatic launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // chunks of ops whose activations come from outside the batch are
    // converted at launch start, chunk i by virtual warp i; they are claimed
    // like the others, so a warp that reaches an op first converts whatever
    // is still unclaimed itself
    for (int i = vw; NTB == 1 && i < a.n_chunks; i += (int)gridDim.x * kCW) {
        int k = 0;
        while (k < a.n_ops && !(a.op[k].f16 && i >= a.op[k].chunk0 && i < a.op[k].chunk0 + a.op[k].n_kc)) ++k;
        if (k == a.n_ops || a.op[k].dseg0 >= 0 || a.op[k].dseg1 >= 0) continue;
        int won = 0;
        if (lane == 0) won = atomicCAS(a.counters + a.op[k].flag_off + (i - a.op[k].chunk0) * kFlagStride, 0, 1) == 0;
        if (__shfl_sync(0xffffffffu, won, 0)) prep_chunk<false>(a, k, i - a.op[k].chunk0, lane);
    }
    if (!has_units) return;

    Walk Wk;
    Wk.slot = 0;
    Wk.parity = 0;
    Wk.n = 0;
    Wk.dead = false;
    int s = 0, gu = 0, gend = 0, k = 0;
    while (!Wk.dead && find_range(a, vw, s, gu, gend)) {
        while (k + 1 < a.n_ops && gu >= a.op[k + 1].ub) ++k;
        const int k_first = k;
        const int rg_first = (gu - a.op[k].ub) / a.op[k].n_kc;
        while (gu < gend && !Wk.dead) {
            const Op& op = a.op[k];
            const int end = min(gend, op.ub + op.units);
            const bool prod = op.dseg0 >= 0 || op.dseg1 >= 0;
            if (prod && op.fed && !(NTB == 1 && op.f16)) {
                // the chunks this warp reads, as the producer writes them
                if (!wait_fed(a, C, k, gu - op.ub, end - op.ub, lane)) {
                    Wk.dead = true;
                    break;
                }
            } else if (prod && !op.fed) {
                // earlier segments whose output this op reads
                bool ok = true;
                if (lane == 0) {
                    if (op.dseg0 >= 0) ok = wait_count(C.seg_done + op.dseg0, a.seg[op.dseg0].active, C.abort, C.err);
                    if (ok && op.dseg1 >= 0)
                        ok = wait_count(C.seg_done + op.dseg1, a.seg[op.dseg1].active, C.abort, C.err);
                }
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                    Wk.dead = true;
                    break;
                }
            }
            bool h = false;
            if constexpr (NTB == 1) {      // the f16 path runs up to 8 tokens
                if (op.f16) {
                    bool bad = false;
                    const bool ok = prod ? ensure_chunks<true>(a, C, k, gu - op.ub, end - op.ub, lane, bad)
                                         : ensure_chunks<false>(a, C, k, gu - op.ub, end - op.ub, lane, bad);
                    if (!ok) {
                        Wk.dead = true;
                        break;
                    }
                    h = !bad;
                }
                if (h)
                    run_op<1, false, true>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring, bars,
                                           s_abort, pair_nv, scale_tab, lane, policy);
            }
            if (h) {
            } else if (prod)
                run_op<NTB, true, false>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring, bars,
                                         s_abort, pair_nv, scale_tab, lane, policy);
            else
                run_op<NTB, false, false>(a, C, F, Wk, s, k, gu, end, gend, vw, k_first, rg_first, ring_p, ring, bars,
                                          s_abort, pair_nv, scale_tab, lane, policy);
            if (((k == a.ar_op && a.ar_world > 0) || op.feed) && !Wk.dead) {
                // the row groups whose first unit lies in [gu, end): this warp wrote them
                const int r_lo = (gu - op.ub + op.n_kc - 1) / op.n_kc, r_hi = (end - 1 - op.ub) / op.n_kc;
                if (r_lo <= r_hi) {
                    if (op.feed)
                        feed_pass(a, k, r_lo, r_hi, lane);
                    else
                        ar_pass(a, C, r_lo, r_hi, lane);
                }
            }
            gu = end;
            if (gu < gend) ++k;
        }
        if (Wk.dead) break;
        // this warp is done with segment s (outputs and partial reads
        // included); the count is kept only for segments something waits on
        if (a.seg[s].waited) {
            __syncwarp();
            if (lane == 0) red_release_add(C.seg_done + s, 1);
        }
        ++s;
    }
    if (Wk.dead) {
        // let the copies in flight land before the CTA retires
        uint32_t sl = Wk.slot, par = Wk.parity;
        for (uint32_t i = Wk.n; i < F.n; ++i) {
            const uint64_t dl = globaltimer_ns() + kWaitNs;
            while (!mbar_try(bars + 8 * sl, par) && globaltimer_ns() < dl) {
            }
            if (++sl == kDepth) {
                sl = 0;
                par ^= 1u;
            }
        }
    }
}

template <int NTB>
__global__ void __launch_bounds__(kThreads, 1) k_stream(const __grid_constant__ Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kCW * kWarpRing);
    uint32_t* pair_nv = reinterpret_cast<uint32_t*>(full + kCW * kDepth);
    uint32_t* scale_tab = pair_nv + 256;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ctl C;
    C.err = reinterpret_cast<int*>(a.ws);
    C.abort = reinterpret_cast<volatile int*>(a.ws + kCtlAbort);
    C.seg_done = reinterpret_cast<int*>(a.ws + kCtlSegDone);
    // the next launch of the stream may start its prologue now (it waits for
    // this grid before it touches anything but its weights)
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) s_abort = 0;
    if (lane == 0) {
        for (int i = 0; i < kDepth; ++i) mbar_init(smem_u32(full + warp * kDepth + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const uint32_t sb = __float_as_uint(e4m3_to_f32((uint32_t)i)) >> 16;   // e4m3 values are exact in bf16
        scale_tab[i] = sb | (sb << 16);
        pair_nv[i] = code_bf16(SPARK_FMT_NVFP4, (uint32_t)i & 15u) | (code_bf16(SPARK_FMT_NVFP4, (uint32_t)i >> 4) << 16);
    }
    __syncthreads();
    // virtual warp: the warps of a CTA take ranges spread over the sequence,
    // so an SM mixes formats (SPFP2 decodes on the integer pipe, FP3 / NVFP4
    // on shared-memory tables and the bf16 multiplier)
    const int vw = warp * (int)gridDim.x + blockIdx.x;
    warp_main<NTB>(a, C, ring + warp * kWarpRing, smem_u32(ring + warp * kWarpRing), smem_u32(full + warp * kDepth),
                   &s_abort, pair_nv, scale_tab, vw, lane);
    __syncthreads();
    // the last CTA out returns the control block to zero for the next launch
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(reinterpret_cast<int*>(a.ws + kCtlCtaDone), 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        const bool aborted = *C.abort != 0;
        for (int i = threadIdx.x; i < a.n_seg; i += blockDim.x) C.seg_done[i] = 0;
        // an aborted launch can leave row-group counters raised; the chunk
        // flags after them are cleared every launch
        for (int i = (aborted ? 0 : a.n_cnt) + threadIdx.x; i < a.n_cnt_all; i += blockDim.x) a.counters[i] = 0;
        __syncthreads();
        if (threadIdx.x == 0) {
            // this rank's count of fused all-reduce calls (the next call's number - 1)
            if (a.ar_world > 0) *a.ar_counter += 1;
            *C.abort = 0;
            __threadfence();
            *reinterpret_cast<volatile int*>(a.ws + kCtlCtaDone) = 0;
        }
    }
}

constexpr size_t kSmemBytes = (size_t)kCW * kWarpRing + (size_t)kCW * kDepth * 8 + (256 + 256) * 4;
static_assert(kSmemBytes <= 227 * 1024, "shared memory above the per-CTA limit");

int sm_count(int dev) {
    static int cache[64] = {};
    if (dev < 0 || dev >= 64) return 0;
    if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
    return cache[dev];
}

std::mutex g_mu;

// cooperative: the batch has several segments, whose waits need every CTA
// resident; otherwise a programmatic launch, which may overlap the previous
// kernel's tail
template <int NTB>
int launch(const Args& a, int grid, cudaStream_t s, bool cooperative) {
    int dev = 0;
    cudaGetDevice(&dev);
    {
        static bool done[64] = {};
        std::lock_guard<std::mutex> lk(g_mu);
        if (!done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(k_stream<NTB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kSmemBytes);
            if (e != cudaSuccess) return set_error((int)e, "k_stream: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (cooperative) {
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_stream<NTB>, a);
    if (e != cudaSuccess) return set_error((int)e, "k_stream launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

}  // namespace stream

// ---------------------------------------------------------------- host entry (used by gemv.cu)
// Workspace layout shared with spark_linear: control block in [0, 4096), the
// row-group counters at `counters_off` (int[max_counters], self-resetting),
// then this kernel's partial sums from `scratch_off`.
struct StreamPlan {
    stream::Args args;
    size_t scratch_bytes = 0;   // bytes needed from scratch_off
    uint8_t* scratch = nullptr; // ws + scratch_off (null for a size query)
    int grid = 0;
};

static int unit_bytes_of(int fmt) {
    return fmt == SPARK_FMT_SPFP2 ? 1280 : (fmt == SPARK_FMT_FP3 ? 1792 : 2304);
}

// Validate a batch and lay it out; ws may be null (size query).
int stream_plan(const SparkChainOp* ops, int n_ops, int64_t M, uint8_t* ws, size_t counters_off,
                int64_t max_counters, size_t scratch_off, StreamPlan* P) {
    using namespace stream;
    SPARK_REQUIRE(ops && n_ops >= 1 && n_ops <= kMaxOps, SPARK_ERR_INVALID,
                  "spark_linear_batch: 1 to %d ops (got %d)", kMaxOps, n_ops);
    SPARK_REQUIRE(M >= 1 && M <= kMaxTok, SPARK_ERR_INVALID, "spark_linear_batch: M must be 1..%d (got %lld)",
                  kMaxTok, (long long)M);
    int dev = 0;
    cudaGetDevice(&dev);
    const int G = sm_count(dev);
    SPARK_REQUIRE(G > 0, SPARK_ERR_DEVICE, "spark_linear_batch: no device");
    const int64_t T = (int64_t)G * kCW;
    Args& a = P->args;
    a = Args{};
    a.n_ops = n_ops;
    a.M = (int)M;
    int64_t cnt = 0, ub = 0;
    int seg_k0 = 0;
    for (int k = 0; k < n_ops; ++k) {
        const SparkChainOp& o = ops[k];
        SPARK_REQUIRE(o.kind == SPARK_CHAIN_LINEAR, SPARK_ERR_UNSUPPORTED,
                      "spark_linear_batch: op %d: only linears (kind %d)", k, o.kind);
        const int flags = o.fmt & ~0xff, fmt = o.fmt & 0xff;
        SPARK_REQUIRE((flags & SPARK_LAYOUT_TILED) && !(flags & ~(SPARK_LAYOUT_TILED | SPARK_EPILOGUE_SILU)),
                      SPARK_ERR_UNSUPPORTED, "spark_linear_batch: op %d: tiled weights (spark_tile_weights) required", k);
        SPARK_REQUIRE(fmt == SPARK_FMT_SPFP2 || fmt == SPARK_FMT_FP3 || fmt == SPARK_FMT_NVFP4, SPARK_ERR_UNSUPPORTED,
                      "spark_linear_batch: op %d: format %d (SPFP2, FP3 or NVFP4)", k, fmt);
        SPARK_REQUIRE(o.wq && o.x && o.y, SPARK_ERR_INVALID, "spark_linear_batch: op %d: null pointer", k);
        SPARK_REQUIRE(o.oc > 0 && o.ic > 0 && o.ic % 256 == 0, SPARK_ERR_INVALID,
                      "spark_linear_batch: op %d: ic must be a positive multiple of 256", k);
        SPARK_REQUIRE(aligned(o.wq, 16) && aligned(o.x, 16) && o.ldx >= o.ic && o.ldx % 8 == 0, SPARK_ERR_ALIGNMENT,
                      "spark_linear_batch: op %d: 16-byte aligned weights and x, ldx a multiple of 8", k);
        const bool silu = (flags & SPARK_EPILOGUE_SILU) != 0;
        SPARK_REQUIRE(!silu || o.oc % 16 == 0, SPARK_ERR_INVALID,
                      "spark_linear_batch: op %d: the fused SiLU takes whole 16-row groups", k);
        SPARK_REQUIRE(o.ldy >= (silu ? o.oc / 2 : o.oc), SPARK_ERR_INVALID, "spark_linear_batch: op %d: ldy", k);
        SPARK_REQUIRE(o.y_dtype >= 0 && o.y_dtype <= 2 && (!o.bias || (o.bias_dtype >= 0 && o.bias_dtype <= 2)),
                      SPARK_ERR_INVALID, "spark_linear_batch: op %d: dtype", k);
        for (int d = 0; d < 2; ++d)
            SPARK_REQUIRE(o.dep[d] >= -1 && o.dep[d] < k, SPARK_ERR_INVALID,
                          "spark_linear_batch: op %d: dep %d must name an earlier op", k, o.dep[d]);
        // an op that reads the output of an op of the current segment opens a new one
        if (o.dep[0] >= seg_k0 || o.dep[1] >= seg_k0) {
            Seg& sg = a.seg[a.n_seg++];
            sg.k0 = seg_k0;
            sg.k1 = k;
            seg_k0 = k;
        }
        Op& p = a.op[k];
        p.w = o.wq;
        p.x = static_cast<const uint16_t*>(o.x);
        p.y = o.y;
        p.bias = o.bias;
        p.ldx = o.ldx;
        p.ldy = o.ldy;
        p.fmt = fmt;
        p.oc = (int)o.oc;
        p.n_kc = (int)(o.ic / 256);
        const int64_t n_rg = (o.oc + 15) / 16;
        const int64_t units = n_rg * p.n_kc;
        SPARK_REQUIRE(units < (1ll << 30) && o.oc < (1ll << 30) && ub + units < (1ll << 31), SPARK_ERR_UNSUPPORTED,
                      "spark_linear_batch: op %d too large", k);
        p.units = (int)units;
        p.ub = (int)ub;
        ub += units;
        p.unit_bytes = unit_bytes_of(fmt);
        p.cnt_off = (int)cnt;
        cnt += n_rg;
        p.seg = a.n_seg;
        p.dseg0 = o.dep[0] >= 0 ? a.op[o.dep[0]].seg : -1;
        p.dseg1 = o.dep[1] >= 0 ? a.op[o.dep[1]].seg : -1;
        p.y_dtype = o.y_dtype;
        p.bias_dtype = o.bias ? o.bias_dtype : 0;
        p.silu = silu ? 1 : 0;
    }
    {
        Seg& sg = a.seg[a.n_seg++];
        sg.k0 = seg_k0;
        sg.k1 = n_ops;
    }
    a.n_cnt = (int)std::min<int64_t>(cnt, max_counters);
    SPARK_REQUIRE(cnt <= max_counters, SPARK_ERR_UNSUPPORTED,
                  "spark_linear_batch: %lld row groups in the batch, above %lld", (long long)cnt, (long long)max_counters);
    // up to 8 tokens, ops take the f16 path while their converted activations
    // fit the budget and their chunk flags fit after the row-group counters
    // (above 8 tokens the per-unit rescaling of two token tiles costs more than
    // the cheaper decode saves)
    int64_t chunks = 0;
    // each chunk flag on its own 128-byte line: every warp that reaches an op
    // claims and polls the flags of the chunks it reads, and flags sharing a
    // line would serialise those atomics and loads in one L2 slice
    const int64_t fbase = (cnt + kFlagStride - 1) / kFlagStride * kFlagStride;
    // (a one-op batch keeps the bf16 path: the conversion's latency at launch
    // start costs more than it saves over the few units each warp then has;
    // so does an all-SPFP2 batch of fewer than kF16Units units per warp, whose
    // bf16 decode is nearly as cheap; with FP3 / NVFP4 ops in the batch the
    // conversion runs anyway and SPFP2 keeps the f16 path too)
    bool all_spfp2 = true;
    for (int k = 0; k < n_ops; ++k) all_spfp2 &= a.op[k].fmt == SPARK_FMT_SPFP2;
    const bool f16_ok = M <= 8 && n_ops > 1 && !(all_spfp2 && ub < (int64_t)kF16Units * T);
    for (int k = 0; k < n_ops && f16_ok; ++k) {
        Op& p = a.op[k];
        if ((size_t)(chunks + p.n_kc) * 512 * M > kXhBudget || fbase + (chunks + p.n_kc) * kFlagStride > max_counters)
            continue;
        p.f16 = 1;
        p.chunk0 = (int)chunks;
        p.flag_off = (int)(fbase + chunks * kFlagStride);
        chunks += p.n_kc;
    }
    // a consumer whose one input is an earlier op's whole bf16 output waits
    // only for the chunks it reads, as the producer's row groups complete (the
    // producer's warp that completes a chunk converts it for an f16 consumer)
    int64_t feeds = fbase + chunks * kFlagStride;
    for (int k = 0; k < n_ops; ++k) {
        Op& c = a.op[k];
        const SparkChainOp& o = ops[k];
        if (o.dep[0] < 0 || o.dep[1] >= 0) continue;
        Op& pr = a.op[o.dep[0]];
        const int width = pr.silu ? pr.oc / 2 : pr.oc;
        if (pr.feed || pr.y != o.x || pr.ldy != c.ldx || pr.y_dtype != SPARK_DTYPE_BF16 || width != c.n_kc * 256 ||
            feeds + (int64_t)c.n_kc * kFlagStride > max_counters)
            continue;
        pr.feed = k + 1;
        pr.feed_rgs = pr.silu ? 32 : 16;
        pr.feed_cnt = (int)feeds;
        c.fed = o.dep[0] + 1;
        feeds += (int64_t)c.n_kc * kFlagStride;
    }
    a.n_cnt_all = (int)(feeds > fbase ? feeds : cnt);
    a.n_chunks = (int)chunks;
    a.part_stride = T * 2 * M * 16;
    const size_t area = (size_t)a.part_stride * sizeof(float);
    a.part_ring = (int)std::max<size_t>(1, std::min<size_t>((size_t)a.n_seg, kPartAreaBudget / area));
    for (int s = 0; s < a.n_seg; ++s) {
        Seg& sg = a.seg[s];
        sg.ub = a.op[sg.k0].ub;
        sg.units = a.op[sg.k1 - 1].ub + a.op[sg.k1 - 1].units - sg.ub;
        sg.q = (int)(sg.units / T);
        sg.rem = (int)(sg.units % T);
        sg.active = sg.q > 0 ? (int)T : sg.rem;
        if (s + a.part_ring < a.n_seg) sg.waited = 1;
    }
    for (int k = 0; k < n_ops; ++k) {
        if (a.op[k].dseg0 >= 0) a.seg[a.op[k].dseg0].waited = 1;
        if (a.op[k].dseg1 >= 0) a.seg[a.op[k].dseg1].waited = 1;
    }
    // scratch: partial-sum areas, then 1 / sigma [chunks][16], then the converted activations
    const size_t inv_off = ((size_t)a.part_ring * area + 255) / 256 * 256;
    const size_t xh_off = inv_off + ((size_t)chunks * 16 * sizeof(float) + 255) / 256 * 256;
    P->scratch_bytes = xh_off + (size_t)chunks * 512 * M;
    P->grid = G;
    a.ws = ws;
    P->scratch = ws ? ws + scratch_off : nullptr;
    if (ws) {
        a.counters = reinterpret_cast<int*>(ws + counters_off);
        a.partials = reinterpret_cast<float*>(ws + scratch_off);
        a.xinv = reinterpret_cast<float*>(ws + scratch_off + inv_off);
        a.xh = reinterpret_cast<uint16_t*>(ws + scratch_off + xh_off);
    }
    return SPARK_OK;
}

// The fused all-reduce of one op of a planned batch (spark_linear_batch_ar):
// the op writes this rank's sums (fp32, no bias) to a scratch buffer, which
// the kernel then exchanges; its real output, bias and dtypes move to Args.
// ar may hold null buffers for a size query.
int stream_plan_set_ar(StreamPlan* P, const SparkBatchAllReduce* ar) {
    using namespace stream;
    Args& a = P->args;
    SPARK_REQUIRE(ar, SPARK_ERR_INVALID, "spark_linear_batch_ar: null all-reduce arguments");
    SPARK_REQUIRE(ar->world >= 1 && ar->world <= SPARK_MAX_PEERS && ar->rank >= 0 && ar->rank < ar->world,
                  SPARK_ERR_INVALID, "spark_linear_batch_ar: rank %d of %d (1 to %d ranks)", ar->rank, ar->world,
                  SPARK_MAX_PEERS);
    SPARK_REQUIRE(ar->op >= 0 && ar->op < a.n_ops, SPARK_ERR_INVALID, "spark_linear_batch_ar: op %d not in the batch",
                  ar->op);
    Op& op = a.op[ar->op];
    SPARK_REQUIRE(!op.silu, SPARK_ERR_UNSUPPORTED, "spark_linear_batch_ar: the all-reduced op cannot fuse SiLU");
    const int nrg = (op.oc + 15) / 16;
    const size_t local_off = (P->scratch_bytes + 255) / 256 * 256;
    P->scratch_bytes = local_off + (size_t)a.M * nrg * 16 * sizeof(float);
    if (!P->scratch) return SPARK_OK;
    SPARK_REQUIRE(ar->recv && ar->counter && aligned(ar->counter, 4), SPARK_ERR_INVALID,
                  "spark_linear_batch_ar: null receive buffers or call counter");
    for (int r = 0; r < ar->world; ++r)
        SPARK_REQUIRE(ar->recv[r] && aligned(ar->recv[r], 16), SPARK_ERR_INVALID,
                      "spark_linear_batch_ar: rank %d's receive buffer missing or misaligned", r);
    for (int r = 0; r < ar->world; ++r) a.ar_recv[r] = static_cast<uint64_t*>(ar->recv[r]);
    a.ar_counter = ar->counter;
    a.ar_world = ar->world;
    a.ar_rank = ar->rank;
    a.ar_nrg = nrg;
    a.ar_op = ar->op;
    a.ar_local = reinterpret_cast<float*>(P->scratch + local_off);
    a.ar_y = op.y;
    a.ar_bias = op.bias;
    a.ar_ldy = op.ldy;
    a.ar_oc = op.oc;
    a.ar_y_dtype = op.y_dtype;
    a.ar_bias_dtype = op.bias_dtype;
    op.y = a.ar_local;
    op.bias = nullptr;
    op.ldy = (int64_t)nrg * 16;
    op.y_dtype = SPARK_DTYPE_F32;
    return SPARK_OK;
}

int stream_plan_alloc(StreamPlan** P) {
    *P = new (std::nothrow) StreamPlan();
    return *P ? SPARK_OK : set_error(SPARK_ERR_INVALID, "spark_linear_batch: out of host memory");
}
void stream_plan_free(StreamPlan* P) { delete P; }
size_t stream_plan_scratch(const StreamPlan* P) { return P->scratch_bytes; }

// scratch of a one-op batch (spark_linear on tiled weights, bf16 x): the
// partial-sum area and the f16 path's converted activations
size_t stream_scratch_single(int64_t M, int64_t ic) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t Mc = M < 1 ? 1 : (M > stream::kMaxTok ? stream::kMaxTok : M);
    const size_t part = (size_t)stream::sm_count(dev) * stream::kCW * 2 * Mc * 16 * sizeof(float);
    size_t bytes = (part + 255) / 256 * 256;
    const int64_t chunks = ic / 256;
    if (Mc <= 8 && (size_t)chunks * 512 * Mc <= stream::kXhBudget)
        bytes += ((size_t)chunks * 16 * sizeof(float) + 255) / 256 * 256 + (size_t)chunks * 512 * Mc;
    return bytes;
}

int stream_launch(const StreamPlan& P, cudaStream_t s) {
    const stream::Args& a = P.args;
    const bool coop = a.n_seg > 1;
    return a.M <= 8 ? stream::launch<1>(a, P.grid, s, coop) : stream::launch<2>(a, P.grid, s, coop);
}

}  // namespace spark
