// gemv.cu -- online-dequant linear for decode-sized batches (M <= 16 per launch).
//
// y[M, oc] = x[M, ic] . decode(W)^T (+ bias) with W in one of the packed SPARK
// formats.  The work is HBM-bound: every packed byte is read exactly once.
//
// Data flow per launch
//   * Decode path (the one layers use): k_gemv_tiled<FMT, NT, XS, BF> on the
//     fragment-major copy made once by spark_tile_weights.  Persistent grid of
//     2 CTAs x 8 warps per SM; every warp owns a contiguous range of "units"
//     (16 rows x 256 columns, 512 for 2:4) in row-group-major order and streams
//     them through a private 4-stage cp.async ring (each lane reads back only
//     the 16-byte vectors it copied).  Each thread decodes two rows straight
//     into MMA A fragments and issues mma.sync m16n8k16 (fp32 accumulate).
//     With bf16 activations every format runs a bf16 MMA on the caller's x
//     (SPFP2 / 2:4 weights are powers of two, FP3 / NVFP4 pairs times an e4m3
//     scale fit bf16 exactly); fp32 / fp16 activations take the fp16 path below.
//   * fp16 path (fp32 / fp16 x, and the reference-layout k_gemv<FMT, NT, XS>):
//     k_prepare_x first writes x as fp16 scaled by a per-token power of two
//     sigma (max|x|/sigma in [2^14, 2^15)), in the column order the format's
//     decoder produces, plus the fp16 remainder of fp32 / fp16 inputs.
//     Products stay exact: every decoded weight has <= 6 significant bits.
//   * Row groups split between warps are reduced deterministically: each
//     contributor writes its fp32 partial to the workspace, bumps a per-row-
//     group counter, and the last arriver sums the partials in warp order.
//   * Optional: the launch requests the next launch's weight into L2
//     (spark_linear_prefetch).
//
// The packed layouts are the reference's (DJAzzs/SPARK 01_core/*_emu.py).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace spark {

namespace {

constexpr int kWarps = 8;         // warps per CTA
constexpr int kDepth = 4;         // ring stages per warp
constexpr int kMaxTokens = 16;    // tokens per launch (NT = 2 MMA n-tiles)
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier wait: 2 s

// ---------------------------------------------------------------- format traits
template <int FMT> struct Fmt;
template <> struct Fmt<SPARK_FMT_SPFP2> {
    static constexpr int kCols = 256;        // columns per unit
    static constexpr int kCodeBytes = 80;    // per row per unit (16 pairs x 5 B)
    static constexpr int kScaleBytes = 0;
    static constexpr int kStride = 80;       // smem row stride (bank-conflict free chunk reads)
    static constexpr int kChunkWords = 5;    // per thread per row
    static constexpr int kSteps = 8;         // 8-column blocks per thread per unit
    // code bits per row: 2.5 per weight
    static int64_t row_bytes(int64_t ic) { return ic / 16 * 5; }
};
template <> struct Fmt<SPARK_FMT_FP3> {
    static constexpr int kCols = 256;
    static constexpr int kCodeBytes = 96;    // 256 x 3 bits
    static constexpr int kScaleBytes = 16;
    static constexpr int kStride = 112;
    static constexpr int kChunkWords = 6;
    static constexpr int kSteps = 8;
    static int64_t row_bytes(int64_t ic) { return ic / 8 * 3; }
};
template <> struct Fmt<SPARK_FMT_NVFP4> {
    static constexpr int kCols = 256;
    static constexpr int kCodeBytes = 128;
    static constexpr int kScaleBytes = 16;
    static constexpr int kStride = 144;
    static constexpr int kChunkWords = 8;
    static constexpr int kSteps = 8;
    static int64_t row_bytes(int64_t ic) { return ic / 2; }
};
template <> struct Fmt<SPARK_FMT_TWOFOUR> {
    static constexpr int kCols = 512;
    static constexpr int kCodeBytes = 112;   // 16 pairs of 16-blocks x 7 B
    static constexpr int kScaleBytes = 0;
    static constexpr int kStride = 112;
    static constexpr int kChunkWords = 7;
    static constexpr int kSteps = 16;
    static int64_t row_bytes(int64_t ic) { return ic / 32 * 7; }
};

// Fragment-major ("tiled") layout: per unit, thread (g, t) owns kFragWords
// words = [chunk of row g][scale word of row g][chunk of row g+8][scale word of
// row g+8]; the unit is stored as kFragWords/4 lane-interleaved 16-byte vectors
// followed by one lane-interleaved 8-byte tail (kFragWords % 4 == 2 for every
// format), so a warp fetches a unit with fully coalesced vector copies.
template <int FMT>
__host__ __device__ constexpr int frag_words() {
    return 2 * (Fmt<FMT>::kChunkWords + (Fmt<FMT>::kScaleBytes ? 1 : 0));
}
template <int FMT>
__host__ __device__ constexpr int unit_bytes_tiled() { return 32 * frag_words<FMT>() * 4; }

template <int FMT>
__host__ __device__ constexpr int stage_bytes() {
    return 16 * Fmt<FMT>::kStride + (Fmt<FMT>::kScaleBytes ? 16 * 16 : 0);
}

// Column permutation inside each 8-column block: position p of the prepared x
// holds original column perm[p].  Decoders emit A registers in this order.
//   kPermNatural  tiled SPFP2 (codes re-ordered at tile time), NVFP4, 2:4
//   kPermSpfp2    SPFP2 in the reference layout: registers hold codes (0,2) (1,3) (4,6) (5,7)
//   kPermFp3      FP3: registers hold codes (0,4) (1,5) (2,6) (3,7)
constexpr int kPermNatural = 0, kPermSpfp2 = 1, kPermFp3 = 2;
__host__ __device__ constexpr int perm_col(int perm, int p) {
    return perm == kPermSpfp2 ? ((p & 4) | ((p & 1) << 1) | ((p >> 1) & 1))
         : perm == kPermFp3 ? ((p & 1) ? 4 + (p >> 1) : (p >> 1)) : p;
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// two e4m3 bytes (low 16 bits of a) -> f16x2, exact
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t a) {
    uint32_t d;
    asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(d) : "r"(a));
    return d;
}

// four bytes of e2m1 pairs -> four f16x2 (byte k -> out[k]; low nibble -> low half)
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t* o) {
    asm("{ .reg .b8 b0, b1, b2, b3;\n"
        "  mov.b32 {b0, b1, b2, b3}, %4;\n"
        "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
        "  cvt.rn.f16x2.e2m1x2 %3, b3; }"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w));
}

__device__ __forceinline__ void mma_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// try_wait with a suspend-time hint: the warp sleeps until the phase completes
// (or ~20 us pass) instead of spinning through issue slots
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

// bounded wait: false once kWaitNs have passed without the phase completing
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t deadline = globaltimer_ns() + kWaitNs;
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() > deadline) return false;
    }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 32-bit window of a little-endian word array starting at bit `pos`
// (pos may be negative: zeros shift in).  pos and N are compile-time.
template <int N>
__device__ __forceinline__ uint32_t window(const uint32_t* c, int pos) {
    if (pos < 0) return c[0] << (-pos);
    const int w = pos >> 5, s = pos & 31;
    if (s == 0) return c[w];
    const uint32_t hi = (w + 1 < N) ? c[w + 1] : 0u;
    return __funnelshift_r(c[w], hi, s);
}

// ---------------------------------------------------------------- decoders
// Each decoder turns step s of a thread's chunk (8 columns of one row) into
// four fp16x2 A registers A[0..3]; A[j] covers prepared columns 2j, 2j+1.

// SPFP2 (block_fp2_emu.py:36, :270-308): value = table(+1,-1,0,0)[code] *
// 2^(e-10).  fp16 of +-2^k has a zero low byte and high byte
// sign | (k+15) << 2, so one byte permute of the block table
// [H, H|0x80, 0, 0] turns four codes (selector nibbles = codes, upper two
// bits clear) into four high bytes; two constant permutes interleave them
// with zero low bytes.  Registers hold codes (0,2) (1,3) (4,6) (5,7).
__device__ __forceinline__ void decode_spfp2(const uint32_t* c, int s, uint32_t* A) {
    const int q = s >> 1, h = s & 1;
    const int P = 40 * q + 16 * h;                     // mantissa bit offset
    const uint32_t e = window<5>(c, 40 * q + 32 + 4 * h) & 0xfu;
    const uint32_t table = e * 0x404u + 0x9414u;       // [(e+5)<<2, ((e+5)<<2)|0x80, 0, 0]
    const uint32_t m = window<5>(c, P);
    const uint32_t he = prmt(table, 0u, m & 0x3333u);          // high bytes of codes 0,2,4,6
    const uint32_t ho = prmt(table, 0u, (m >> 2) & 0x3333u);   // codes 1,3,5,7
    A[0] = prmt(he, 0u, 0x1404u);
    A[1] = prmt(ho, 0u, 0x1404u);
    A[2] = prmt(he, 0u, 0x3424u);
    A[3] = prmt(ho, 0u, 0x3424u);
}

// FP3 (fp3_emu.py:47, :142-154): 8 codes of a 24-bit group, code i at bits 3i;
// unscaled fp16 high bytes of (0,.5,1,1.5,-0,-.5,-1,-1.5) form an 8-byte table
// (low bytes are zero), then one f16x2 multiply applies the e4m3 scale.
__device__ __forceinline__ void decode_fp3(const uint32_t* c, uint32_t scale_word, int s, uint32_t* A) {
    const uint32_t v = window<6>(c, 24 * s) & 0xffffffu;
    const uint32_t sb = (scale_word >> (8 * (s >> 1))) & 0xffu;
    const uint32_t s2 = e4m3x2_to_f16x2(sb * 0x101u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t sel = (((v >> (3 * j)) & 7u) << 4) | (((v >> (3 * j + 12)) & 7u) << 12);
        A[j] = hmul2(prmt(0x3e3c3800u, 0xbebcb880u, sel), s2);
    }
}

// NVFP4 (nvfp4_emu.py:109-123): codes are standard e2m1 nibbles (element 2k in
// the low nibble); the hardware converter gives exact fp16, then the scale.
__device__ __forceinline__ void decode_nvfp4(const uint32_t* c, uint32_t scale_word, int s, uint32_t* A) {
    const uint32_t sb = (scale_word >> (8 * (s >> 1))) & 0xffu;
    const uint32_t s2 = e4m3x2_to_f16x2(sb * 0x101u);
    uint32_t u[4];
    e2m1x8_to_f16x2(c[s], u);
#pragma unroll
    for (int j = 0; j < 4; ++j) A[j] = hmul2(u[j], s2);
}

// FP3 / NVFP4 for a bf16 MMA on the caller's bf16 x (no prepared copy): the
// natural column pair (2j, 2j+1) is one field of the packed codes -- FP3 the
// 6 bits at 6j of the step's 24-bit group, NVFP4 byte j of the step's word --
// and indexes a shared-memory table of unscaled bf16x2 values; one bf16x2
// multiply by the block's e4m3 scale (also tabled as bf16x2) finishes the
// pair.  Exact: an FP3 / e2m1 value has at most 2 significant bits, an e4m3
// scale at most 4, so every product fits bf16's 8.
template <int FMT>
__device__ __forceinline__ void decode_scaled_bf16(const uint32_t* c, uint32_t scale_word, int s,
                                                   const uint32_t* pair_tab, const uint32_t* scale_tab, uint32_t* A) {
    const uint32_t s2 = scale_tab[(scale_word >> (8 * (s >> 1))) & 0xffu];
    if constexpr (FMT == SPARK_FMT_FP3) {
        const uint32_t v = window<6>(c, 24 * s);
#pragma unroll
        for (int j = 0; j < 4; ++j) A[j] = bmul2(pair_tab[(v >> (6 * j)) & 63u], s2);
    } else {
        const uint32_t v = c[s];
#pragma unroll
        for (int j = 0; j < 4; ++j) A[j] = bmul2(pair_tab[(v >> (8 * j)) & 0xffu], s2);
    }
}

// bf16 bits of an FP3 (3-bit) or e2m1 (4-bit) code: sign in the top bit,
// magnitudes 0, .5, 1, 1.5 (FP3) or 0, .5, 1, 1.5, 2, 3, 4, 6 (e2m1)
__device__ __forceinline__ uint32_t code_bf16(int fmt, uint32_t code) {
    const int bits = fmt == SPARK_FMT_FP3 ? 3 : 4;
    const uint32_t mag = code & ((1u << (bits - 1)) - 1u), neg = code >> (bits - 1);
    const float tab[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    return (__float_as_uint(tab[mag]) >> 16) | (neg << 15);
}

// 2:4 SPFP2 (two_four.py:158-189): 28-bit slot per 16-block, 4 groups of 4
// columns with a 4-bit position mode and two sign bits (decode_twofour_t).
// bf16 variants for SPFP2 and 2:4 (weights +-2^(e-10), e in [0,15]).  bf16 of
// +-2^k has biased exponent E = 117 + e: high byte sign | E >> 1, low byte
// (E & 1) << 7.  A 16-entry shared-memory table holds, per e, the byte tables
// [H, H|0x80, 0, 0] and [L, L, 0, 0]; the tiled layout stores each mantissa
// word with codes (1,2) and (5,6) swapped so the registers come out in
// natural column order (0,1) (2,3) (4,5) (6,7).
__device__ __forceinline__ void decode_spfp2_bf16(const uint32_t* c, int s, const uint2* lut, uint32_t* A) {
    const int q = s >> 1, h = s & 1;
    const int P = 40 * q + 16 * h;
    const uint2 tab = *reinterpret_cast<const uint2*>(
        reinterpret_cast<const uint8_t*>(lut) + (window<5>(c, 40 * q + 32 + 4 * h - 3) & 0x78u));
    const uint32_t m = window<5>(c, P);
    const uint32_t se = m & 0x3333u, so = (m >> 2) & 0x3333u;
    const uint32_t he = prmt(tab.x, 0u, se), ho = prmt(tab.x, 0u, so);
    const uint32_t le = prmt(tab.y, 0u, se), lo = prmt(tab.y, 0u, so);
    A[0] = prmt(le, he, 0x5140u);
    A[1] = prmt(lo, ho, 0x5140u);
    A[2] = prmt(le, he, 0x7362u);
    A[3] = prmt(lo, ho, 0x7362u);
}

__device__ __forceinline__ uint32_t tf_val(uint32_t H16, uint32_t mode, uint32_t sg, int p) {
    int a = -1, b = -1;
    if (mode < 6u) {
        a = mode < 3u ? 0 : (mode < 5u ? 1 : 2);
        b = mode == 0u ? 1 : (mode == 1u ? 2 : ((mode == 2u || mode == 4u || mode == 5u) ? 3 : 2));
    } else if (mode >= 8u && mode <= 11u) {
        a = (int)mode - 8;
    }
    if (p == a) return H16 | ((sg & 1u) << 15);
    if (p == b) return H16 | ((sg >> 1) << 15);
    return 0u;
}

// 2:4 with either fp16 or bf16 magnitude bits
template <bool BF>
__device__ __forceinline__ void decode_twofour_t(const uint32_t* c, int s, uint32_t* A) {
    const int q = s >> 2, slot = (s >> 1) & 1, half = s & 1;
    const uint32_t w = window<7>(c, 56 * q + 28 * slot) & 0x0fffffffu;
    const uint32_t e = (w >> 24) & 0xfu;
    const uint32_t H16 = BF ? (117u + e) << 7 : (e + 5u) << 10;
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
        const int g = 2 * half + gg;
        const uint32_t mode = (w >> (4 * g)) & 0xfu;
        const uint32_t sg = (w >> (16 + 2 * g)) & 3u;
        A[2 * gg] = tf_val(H16, mode, sg, 0) | (tf_val(H16, mode, sg, 1) << 16);
        A[2 * gg + 1] = tf_val(H16, mode, sg, 2) | (tf_val(H16, mode, sg, 3) << 16);
    }
}

__device__ __forceinline__ void mma_16816_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int FMT>
__device__ __forceinline__ void decode_step(const uint32_t* c, uint32_t sw, int s, uint32_t* A) {
    if constexpr (FMT == SPARK_FMT_SPFP2) decode_spfp2(c, s, A);
    else if constexpr (FMT == SPARK_FMT_FP3) decode_fp3(c, sw, s, A);
    else if constexpr (FMT == SPARK_FMT_NVFP4) decode_nvfp4(c, sw, s, A);
    else decode_twofour_t<false>(c, s, A);
}

// Sum, in warp order, of the partials that warps w_lo..w_hi published for
// one row group.  Warps after w_lo start inside the row group, so they hold
// it in slot 0; w_lo holds it in slot 1 when its range began in an earlier
// row group.  A batch's loads are all issued before its first add: the
// reduction costs one L2 round trip per batch instead of one per warp.
template <int NT>
__device__ __forceinline__ void sum_partials(const float* partials, int w_lo, int w_hi, bool lo_second, int lane,
                                             float (&sum)[NT][4]) {
    constexpr int B = 8 / NT;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sum[nt][i] = 0.0f;
    for (int w0 = w_lo; w0 <= w_hi; w0 += B) {
        float4 v[B][NT];
#pragma unroll
        for (int k = 0; k < B; ++k) {
            const int w = w0 + k;
            const int sl = (w == w_lo && lo_second) ? 1 : 0;
            const float4* src = reinterpret_cast<const float4*>(partials + (((int64_t)w * 2 + sl) * NT * 32 + lane) * 4);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) v[k][nt] = w <= w_hi ? __ldcg(src + nt * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < B; ++k) {
            if (w0 + k > w_hi) break;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                sum[nt][0] += v[k][nt].x; sum[nt][1] += v[k][nt].y; sum[nt][2] += v[k][nt].z; sum[nt][3] += v[k][nt].w;
            }
        }
    }
}

// ---------------------------------------------------------------- kernel args
struct GemvArgs {
    const uint8_t* wq;
    const uint8_t* scales;
    const __half* xp;       // prepared x [M][ic] (fp16, permuted)
    const void* x_raw;      // caller's bf16 x (kernels that stage x themselves)
    int64_t ldx;
    const float* sigma;     // [M] per-token scale of xp
    const void* bias;
    void* y;
    float* partials;        // [T][2][NT*32*4]
    int* counters;          // [n_rg]
    int* err;
    int64_t oc, ic, ldy;
    int64_t row_bytes, scale_row_bytes;
    int64_t n_rg, n_kc, units;
    int M, bias_dtype, y_dtype;
    const uint8_t* pf;      // bytes the next launch will read (L2 prefetch hint), or null
    int64_t pf_bytes;
    int silu_pairs;         // rows 16k..16k+7 gate, 16k+8.. up: write SiLU(gate) * up, oc / 2 columns
};

// ---------------------------------------------------------------- prepare x
// grid = M blocks of kPrepThreads.  sigma = 2^(floor(log2 max|x|) - 14) (1 when
// x is all zero or has a non-finite value); xp[m][8b + p] =
// fp16(x[m][8b + perm[p]] / sigma), and with `split` xp[16 + m][.] holds the
// fp16 remainder (fp32 / fp16 activations carry more bits than one fp16 after
// scaling).  One pass: each thread keeps its 8-element blocks in registers
// between the max reduction and the conversion.
constexpr int kPrepThreads = 512;
constexpr int kPrepBlocks = 4;   // 8-element blocks per thread kept in registers

__device__ __forceinline__ void load8(const void* x, int dt, int64_t off, float* v) {
    if (dt == SPARK_DTYPE_BF16 || dt == SPARK_DTYPE_F16) {
        const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (dt == SPARK_DTYPE_BF16) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            } else {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                v[2 * i] = f.x;
                v[2 * i + 1] = f.y;
            }
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + off + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

__global__ void __launch_bounds__(kPrepThreads) k_prepare_x(const void* __restrict__ x, int x_dtype, int64_t ldx,
                                                            int64_t ic, int fmt, __half* __restrict__ xp,
                                                            float* __restrict__ sigma, int split) {
    // launched as a programmatic dependent of the previous kernel on the stream:
    // x may be that kernel's output, so wait for it before reading; let the
    // GEMV that consumes this kernel's output launch right away
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float red[kPrepThreads / 32];
    __shared__ int bad[kPrepThreads / 32];
    const int m = blockIdx.x;
    const int64_t row = (int64_t)m * ldx;
    const int64_t nblk = ic / 8;
    const bool vec = ((ldx & 7) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    float v[kPrepBlocks][8];
    float mx = 0.0f;
    int nonfinite = 0;
#pragma unroll
    for (int k = 0; k < kPrepBlocks; ++k) {
        const int64_t b = threadIdx.x + (int64_t)k * kPrepThreads;
        if (b < nblk) {
            if (vec) load8(x, x_dtype, row + 8 * b, v[k]);
            else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[k][i] = load_as_float(x, x_dtype, row + 8 * b + i);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float a = fabsf(v[k][i]);
                nonfinite |= !(a <= 3.4028235e38f);
                mx = fmaxf(mx, a);
            }
        }
    }
    // columns beyond kPrepBlocks * kPrepThreads * 8 (very wide layers): second pass
    for (int64_t b = threadIdx.x + (int64_t)kPrepBlocks * kPrepThreads; b < nblk; b += kPrepThreads)
        for (int i = 0; i < 8; ++i) {
            const float a = fabsf(load_as_float(x, x_dtype, row + 8 * b + i));
            nonfinite |= !(a <= 3.4028235e38f);
            mx = fmaxf(mx, a);
        }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
    }
    if ((threadIdx.x & 31) == 0) { red[threadIdx.x >> 5] = mx; bad[threadIdx.x >> 5] = nonfinite; }
    __syncthreads();
    float gmx = 0.0f;
    int gbad = 0;
#pragma unroll
    for (int i = 0; i < kPrepThreads / 32; ++i) { gmx = fmaxf(gmx, red[i]); gbad |= bad[i]; }
    int k2 = 0;
    if (!gbad && gmx > 0.0f) {
        int e;
        frexpf(gmx, &e);            // gmx = f * 2^e, f in [0.5, 1)
        k2 = (e - 1) - 14;
        k2 = k2 < -100 ? -100 : (k2 > 100 ? 100 : k2);
    }
    const float inv = ldexpf(1.0f, -k2);
    if (threadIdx.x == 0) sigma[m] = ldexpf(1.0f, k2);
    auto emit = [&](int64_t b, const float* vb) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 8; p += 2) {
            const float a0 = vb[perm_col(fmt, p)] * inv, a1 = vb[perm_col(fmt, p + 1)] * inv;  // fmt = perm id
            const __half2 h2 = __floats2half2_rn(a0, a1);
            hi[p / 2] = *reinterpret_cast<const uint32_t*>(&h2);
            const float2 back = __half22float2(h2);
            const __half2 l2 = __floats2half2_rn(a0 - back.x, a1 - back.y);
            lo[p / 2] = *reinterpret_cast<const uint32_t*>(&l2);
        }
        *reinterpret_cast<uint4*>(xp + (int64_t)m * ic + 8 * b) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (split)
            *reinterpret_cast<uint4*>(xp + (int64_t)(kMaxTokens + m) * ic + 8 * b) =
                make_uint4(lo[0], lo[1], lo[2], lo[3]);
    };
#pragma unroll
    for (int k = 0; k < kPrepBlocks; ++k) {
        const int64_t b = threadIdx.x + (int64_t)k * kPrepThreads;
        if (b < nblk) emit(b, v[k]);
    }
    for (int64_t b = threadIdx.x + (int64_t)kPrepBlocks * kPrepThreads; b < nblk; b += kPrepThreads) {
        float vb[8];
        for (int i = 0; i < 8; ++i) vb[i] = load_as_float(x, x_dtype, row + 8 * b + i);
        emit(b, vb);
    }
}

// ---------------------------------------------------------------- epilogue
template <int NT>
__device__ __forceinline__ void write_rows(const GemvArgs& a, int64_t rg, const float (*acc)[4], int lane,
                                           const float* sig) {
    const int g = lane >> 2, t = lane & 3;
    if (a.silu_pairs) {
        // this thread holds gate row 16rg+g (acc[.][0..1]) and its up row
        // 16rg+g+8 (acc[.][2..3]): h[tok, 8rg+g] = SiLU(gate) * up
        const int64_t rgate = rg * 16 + g, rup = rgate + 8;
        const float bg = a.bias ? load_as_float(a.bias, a.bias_dtype, rgate) : 0.0f;
        const float bu = a.bias ? load_as_float(a.bias, a.bias_dtype, rup) : 0.0f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int tok = nt * 8 + 2 * t + i;
                if (tok < a.M) {
                    const float s = sig ? sig[tok] : 1.0f;
                    const float gv = (sig ? acc[nt][i] * s : acc[nt][i]) + bg;
                    const float uv = (sig ? acc[nt][2 + i] * s : acc[nt][2 + i]) + bu;
                    store_from_float(a.y, a.y_dtype, (int64_t)tok * a.ldy + rg * 8 + g,
                                     gv / (1.0f + __expf(-gv)) * uv);
                }
            }
        return;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = nt * 8 + 2 * t + (i & 1);
            const int64_t row = rg * 16 + g + ((i >> 1) ? 8 : 0);
            if (tok < a.M && row < a.oc) {
                float v = sig ? acc[nt][i] * sig[tok] : acc[nt][i];
                if (a.bias) v += load_as_float(a.bias, a.bias_dtype, row);
                store_from_float(a.y, a.y_dtype, (int64_t)tok * a.ldy + row, v);
            }
        }
    }
}

// ---------------------------------------------------------------- main kernel
template <int FMT, int NT, int XS>
__global__ void __launch_bounds__(kWarps * 32, 2) k_gemv(const GemvArgs a) {
    using F = Fmt<FMT>;
    constexpr int SB = stage_bytes<FMT>();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem + warp * kDepth * SB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kDepth * SB) + warp * kDepth;

    // all unit bookkeeping in 32-bit integers (units < 2^31 is checked on the host)
    const int T = (int)gridDim.x * kWarps;
    const int gw = (int)blockIdx.x * kWarps + warp;
    const int U = (int)a.units, nkc = (int)a.n_kc;
    const int u0 = (int)((int64_t)U * gw / T), u1 = (int)((int64_t)U * (gw + 1) / T);
    const int n = u1 - u0;

    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kDepth; ++i) mbar_init(smem_addr(bars + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    // producer cursor: (rg, kc) of the next unit to copy
    int prg = u0 / nkc, pkc = u0 - prg * nkc;
    const uint8_t* wrow = a.wq + ((int64_t)prg * 16 + (lane & 15)) * a.row_bytes;
    const uint8_t* srow = a.scales + ((int64_t)prg * 16 + (lane & 15)) * a.scale_row_bytes;
    auto issue = [&](int st) {
        const int rows = min(16, (int)(a.oc - (int64_t)prg * 16));
        const uint32_t bar = smem_addr(bars + st);
        if (lane == 0) mbar_expect_tx(bar, (uint32_t)(rows * (F::kCodeBytes + F::kScaleBytes)));
        __syncwarp();
        uint8_t* dst = ring + st * SB;
        if (lane < 16) {
            if (lane < rows)
                bulk_g2s(smem_addr(dst + lane * F::kStride), wrow + pkc * F::kCodeBytes, F::kCodeBytes, bar);
        } else if (F::kScaleBytes) {
            if (lane - 16 < rows)
                bulk_g2s(smem_addr(dst + 16 * F::kStride + (lane - 16) * 16), srow + pkc * 16, 16, bar);
        }
        if (++pkc == nkc) {
            pkc = 0;
            ++prg;
            wrow += 16 * a.row_bytes;
            srow += 16 * a.scale_row_bytes;
        }
    };

    for (int i = 0; i < kDepth && i < n; ++i) issue(i);
    // the next kernel on the stream may launch now and stage its own weights;
    // it waits (griddepcontrol.wait) for this grid before touching shared data
    asm volatile("griddepcontrol.launch_dependents;");

    // x is produced by k_prepare_x; wait for it (programmatic dependent launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;

    const __half* xrow0 = a.xp + (int64_t)g * a.ic + t * (F::kCols / 4);
    const __half* xrow1 = a.xp + (int64_t)(g + 8) * a.ic + t * (F::kCols / 4);
    const bool tok0 = g < a.M, tok1 = (g + 8) < a.M;
    const int rg_first = u0 / nkc;

    auto flush = [&](int rg, int seg0, int seg1) {
        if (seg0 == rg * nkc && seg1 == (rg + 1) * nkc) {
            write_rows<NT>(a, rg, acc, lane, a.sigma);
            return;
        }
        // partial row group: publish, count, last arriver reduces in warp order
        const int slot = (rg == rg_first) ? 0 : 1;
        float* mine = a.partials + (((int64_t)gw * 2 + slot) * NT * 32 + lane) * 4;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            __stcg(reinterpret_cast<float4*>(mine + nt * 128), make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
        __threadfence();
        __syncwarp();
        // contributors: owners of the first and last unit of the row group
        const int64_t first = (int64_t)rg * nkc, last = (int64_t)(rg + 1) * nkc - 1;
        const int w_lo = (int)(((first + 1) * T - 1) / U), w_hi = (int)(((last + 1) * T - 1) / U);
        int old = 0;
        if (lane == 0) old = atomicAdd(a.counters + rg, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != w_hi - w_lo) return;
        __threadfence();
        float sum[NT][4];
        const bool lo_second = (int)((int64_t)U * w_lo / T) / nkc != rg;
        sum_partials<NT>(a.partials, w_lo, w_hi, lo_second, lane, sum);
        write_rows<NT>(a, rg, sum, lane, a.sigma);
        if (lane == 0) a.counters[rg] = 0;
    };

    // consumer cursor
    int crg = rg_first, ckc = u0 - rg_first * nkc;
    int seg0 = u0;
    for (int i = 0; i < n; ++i) {
        const int st = i % kDepth;
        const uint32_t parity = (uint32_t)((i / kDepth) & 1);
        const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_addr(bars + st), parity));
        if (!ok) {
            if (lane == 0) report_device_error(a.err, 1);
            // let the copies already issued land before the CTA retires
            for (int j = i + 1; j < min(n, i + kDepth); ++j)
                mbar_wait(smem_addr(bars + (j % kDepth)), (uint32_t)((j / kDepth) & 1));
            return;
        }
        // this thread's chunk of rows g and g+8
        const uint8_t* stage = ring + st * SB;
        uint32_t c0[F::kChunkWords], c1[F::kChunkWords];
        const uint32_t* r0 = reinterpret_cast<const uint32_t*>(stage + g * F::kStride) + t * F::kChunkWords;
        const uint32_t* r1 = reinterpret_cast<const uint32_t*>(stage + (g + 8) * F::kStride) + t * F::kChunkWords;
#pragma unroll
        for (int k = 0; k < F::kChunkWords; ++k) { c0[k] = r0[k]; c1[k] = r1[k]; }
        uint32_t sw0 = 0, sw1 = 0;
        if constexpr (F::kScaleBytes != 0) {
            const uint32_t* sc = reinterpret_cast<const uint32_t*>(stage + 16 * F::kStride);
            sw0 = sc[g * 4 + t];
            sw1 = sc[(g + 8) * 4 + t];
        }
        // the stage must be fully read into registers before the bulk copy of
        // unit i + kDepth overwrites it: consume every loaded word, then sync
#pragma unroll
        for (int k = 0; k < F::kChunkWords; ++k) asm volatile("" ::"r"(c0[k]), "r"(c1[k]));
        asm volatile("" ::"r"(sw0), "r"(sw1));
        __syncwarp();
        if (i + kDepth < n) issue(st);

        const int64_t col0 = (int64_t)ckc * F::kCols;
#pragma unroll
        for (int s = 0; s < F::kSteps; ++s) {
            uint32_t A0[4], A1[4];
            decode_step<FMT>(c0, sw0, s, A0);
            decode_step<FMT>(c1, sw1, s, A1);
#pragma unroll
            for (int part = 0; part < XS; ++part) {
                const int64_t po = (int64_t)part * kMaxTokens * a.ic + col0 + 8 * s;
                uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
                if (tok0) x0 = ldg_nc_v4(xrow0 + po);
                if (NT > 1 && tok1) x1 = ldg_nc_v4(xrow1 + po);
                mma_16816(acc[0], A0[0], A1[0], A0[1], A1[1], x0.x, x0.y);
                mma_16816(acc[0], A0[2], A1[2], A0[3], A1[3], x0.z, x0.w);
                if (NT > 1) {
                    mma_16816(acc[NT - 1], A0[0], A1[0], A0[1], A1[1], x1.x, x1.y);
                    mma_16816(acc[NT - 1], A0[2], A1[2], A0[3], A1[3], x1.z, x1.w);
                }
            }
        }
        // advance the consumer cursor; flush at the end of a row group
        const int u = u0 + i;
        if (++ckc == nkc || i + 1 == n) {
            flush(crg, seg0, u + 1);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[nt][q] = 0.0f;
            if (ckc == nkc) { ckc = 0; ++crg; }
            seg0 = u + 1;
        }
    }
}

// ---------------------------------------------------------------- tiled layout
// FP3 code words of one row's 64-column chunk.  Reference packing (six
// words): code k at bit 3k (magnitude bits 0-1, sign bit 2, fp3_emu.py:107).
// Tiled packing: two groups of three words; in group q, nibble i of word j
// (j < 3) is code 32q + 8j + i as an e2m1 code (magnitude bits 0-1, sign bit
// 3: FP3's magnitudes {0, .5, 1, 1.5} are e2m1's codes 0-3), and bit 2 of
// nibble i of words 0, 1, 2 holds bit 0, 1, 2 of code 32q + 24 + i.
__host__ __device__ inline uint32_t fp3_code(const uint32_t* ref, int k) {
    const int b = 3 * k, w = b >> 5, o = b & 31;
    uint32_t v = ref[w] >> o;
    if (o > 29) v |= ref[w + 1] << (32 - o);
    return v & 7u;
}
__host__ __device__ inline void fp3_pack_tiled(const uint32_t* ref, uint32_t* out) {
    for (int q = 0; q < 2; ++q)
        for (int j = 0; j < 3; ++j) {
            uint32_t w = 0;
            for (int i = 0; i < 8; ++i) {
                const uint32_t c = fp3_code(ref, 32 * q + 8 * j + i), x = fp3_code(ref, 32 * q + 24 + i);
                w |= ((c & 3u) | ((x >> j) & 1u) << 2 | (c >> 2) << 3) << (4 * i);
            }
            out[3 * q + j] = w;
        }
}
__device__ inline void fp3_unpack_tiled(const uint32_t* in, uint32_t* ref) {
#pragma unroll
    for (int w = 0; w < 6; ++w) ref[w] = 0u;
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t c;
                if (j < 3) {
                    const uint32_t n = in[3 * q + j] >> (4 * i);
                    c = (n & 3u) | ((n >> 1) & 4u);
                } else {
                    c = ((in[3 * q] >> (4 * i + 2)) & 1u) | (((in[3 * q + 1] >> (4 * i + 2)) & 1u) << 1) |
                        (((in[3 * q + 2] >> (4 * i + 2)) & 1u) << 2);
                }
                const int b = 3 * (32 * q + 8 * j + i);
                ref[b >> 5] |= c << (b & 31);
                if ((b & 31) > 29) ref[(b >> 5) + 1] |= c >> (32 - (b & 31));
            }
        }
}

// thread = (unit, lane): gather the lane's fragment words from the reference
// layout and store them in fragment-major order
template <int FMT>
__global__ void __launch_bounds__(256) k_tile(const uint8_t* __restrict__ wq, const uint8_t* __restrict__ scales,
                                              int64_t oc, int64_t row_bytes, int64_t scale_row_bytes, int64_t n_kc,
                                              int64_t units, uint8_t* __restrict__ tiled) {
    using F = Fmt<FMT>;
    constexpr int FW = frag_words<FMT>();
    constexpr int NV = FW / 4;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t u = idx >> 5;
    const int lane = (int)(idx & 31);
    if (u >= units) return;
    const int64_t rg = u / n_kc, kc = u - rg * n_kc;
    const int g = lane >> 2, t = lane & 3;
    uint32_t w[FW];
    int k = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int64_t row = rg * 16 + g + 8 * half;
        const bool ok = row < oc;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(wq + row * row_bytes + kc * F::kCodeBytes) +
                              t * F::kChunkWords;
#pragma unroll
        for (int j = 0; j < F::kChunkWords; ++j) {
            uint32_t v = 0u;
            if (ok) v = src[j];
            w[k++] = v;
        }
        if constexpr (F::kScaleBytes != 0) {
            uint32_t v = 0u;
            if (ok) v = reinterpret_cast<const uint32_t*>(scales + row * scale_row_bytes + kc * 16)[t];
            w[k++] = v;
        }
    }
    if constexpr (FMT == SPARK_FMT_SPFP2) {
        // Stream layout (the decoders of stream.cu): per 8-column block s of
        // the chunk, word s holds the 16 codes of rows g and g + 8 so that
        // (word >> 2j) & 0x03030303 has, byte by byte, the codes of columns
        // 2j and 2j + 1 of row g, then of row g + 8; words 8-9: byte s % 4 of
        // word 8 + s / 4 = e(row g) | e(row g + 8) << 4.  The reference pair
        // layout holds, per 16 columns, mantissa words m0, m1 (column j at
        // bits 2j) and the exponent byte e0 | e1 << 4.
        const uint8_t* b = reinterpret_cast<const uint8_t*>(w);
        uint32_t out[10] = {};
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int blk = 0; blk < 8; ++blk) {
                const uint8_t* q = b + half * 20 + (blk >> 1) * 5;
                const int h = blk & 1;
                const uint32_t m = (uint32_t)q[2 * h] | ((uint32_t)q[2 * h + 1] << 8);
                const uint32_t e = h ? (q[4] >> 4) : (q[4] & 0xfu);
                uint32_t p = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) p |= ((m >> (2 * i)) & 3u) << (2 * (i >> 1) + 8 * (i & 1) + 16 * half);
                out[blk] |= p;
                out[8 + (blk >> 2)] |= e << (8 * (blk & 3) + 4 * half);
            }
#pragma unroll
        for (int i = 0; i < 10; ++i) w[i] = out[i];
    }
    if constexpr (FMT == SPARK_FMT_FP3) {
        // per row: six code words re-packed for the e2m1 conversion, then the scale word
        uint32_t out[6];
        fp3_pack_tiled(w, out);
        for (int i = 0; i < 6; ++i) w[i] = out[i];
        fp3_pack_tiled(w + 7, out);
        for (int i = 0; i < 6; ++i) w[7 + i] = out[i];
    }
    uint8_t* dst = tiled + u * unit_bytes_tiled<FMT>();
#pragma unroll
    for (int v = 0; v < NV; ++v)
        reinterpret_cast<uint4*>(dst)[v * 32 + lane] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    reinterpret_cast<uint2*>(dst + NV * 512)[lane] = make_uint2(w[4 * NV], w[4 * NV + 1]);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// GEMV over tiled weights.  Every thread copies its own fragment vectors of
// the next kDepthT units into a private shared-memory ring (cp.async), so no
// synchronisation beyond the thread's own wait_group is needed.
constexpr int kDepthT = 4;
constexpr int64_t kPrefetchChunk = 32 * 1024;   // bytes per L2 prefetch instruction

// acquire-release counter bump: the partials written before it are visible to
// whoever observes the count, and the last arriver sees everybody's partials
__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// BF: bf16 MMA with the caller's bf16 x read directly (SPFP2 and 2:4, whose
// weights are exact in bf16); otherwise fp16 MMA on the prepared x.
template <int FMT, int NT, int XS, bool BF>
__global__ void __launch_bounds__(kWarps * 32, 2) k_gemv_tiled(const GemvArgs a) {
    using F = Fmt<FMT>;
    constexpr int FW = frag_words<FMT>();
    constexpr int NV = FW / 4;
    constexpr int UB = unit_bytes_tiled<FMT>();

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint2 lut[16];
    __shared__ uint32_t pair_tab[FMT == SPARK_FMT_FP3 || FMT == SPARK_FMT_NVFP4 ? 256 : 1];
    __shared__ uint32_t scale_tab[FMT == SPARK_FMT_FP3 || FMT == SPARK_FMT_NVFP4 ? 256 : 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // ring slot (stage, vector) of this thread: 16 bytes each
    uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * kDepthT * (NV + 1) * 32 + lane;

    const int T = (int)gridDim.x * kWarps;
    const int gw = (int)blockIdx.x * kWarps + warp;
    const int U = (int)a.units, nkc = (int)a.n_kc;
    const int u0 = (int)((int64_t)U * gw / T), u1 = (int)((int64_t)U * (gw + 1) / T);
    const int n = u1 - u0;

    auto issue = [&](int u, int st) {
        if (u < u1) {
            const uint8_t* src = a.wq + (int64_t)u * UB;
            uint4* dst = ring + st * (NV + 1) * 32;
#pragma unroll
            for (int v = 0; v < NV; ++v) cp_async16(smem_addr(dst + v * 32), src + (v * 32 + lane) * 16);
            cp_async8(smem_addr(dst + NV * 32), src + NV * 512 + lane * 8);
        }
        cp_async_commit();
    };
    // Hint for the next launch: this CTA's share of the bytes it will read
    // goes to L2 now, streaming from DRAM while this launch decodes.
    if (a.pf && threadIdx.x == 0) {
        const int64_t g = a.pf_bytes / 16;
        const int64_t g0 = g * blockIdx.x / gridDim.x, g1 = g * (blockIdx.x + 1) / gridDim.x;
        for (int64_t c = g0; c < g1; c += kPrefetchChunk / 16) {
            const int64_t left = g1 - c;
            const uint32_t bytes = (uint32_t)(left < kPrefetchChunk / 16 ? left : kPrefetchChunk / 16) * 16u;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf + c * 16), "r"(bytes) : "memory");
        }
    }
#pragma unroll
    for (int i = 0; i < kDepthT; ++i) issue(u0 + i, i);
    if constexpr (BF && FMT == SPARK_FMT_SPFP2) {
        if (threadIdx.x < 16) {
            const uint32_t E = 117u + threadIdx.x;
            const uint32_t H = E >> 1, L = (E & 1u) << 7;
            lut[threadIdx.x] = make_uint2(H * 0x101u + 0x8000u, L * 0x101u);
        }
        __syncthreads();
    }
    if constexpr (BF && (FMT == SPARK_FMT_FP3 || FMT == SPARK_FMT_NVFP4)) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) {
            // e4m3 values are exact in bf16: the top half of the fp32 bits
            const uint32_t sb = __float_as_uint(e4m3_to_f32((uint32_t)i)) >> 16;
            scale_tab[i] = sb | (sb << 16);
            const int bits = FMT == SPARK_FMT_FP3 ? 3 : 4;
            if (i < (1 << (2 * bits)))
                pair_tab[i] = code_bf16(FMT, (uint32_t)i & ((1u << bits) - 1u)) |
                              (code_bf16(FMT, (uint32_t)i >> bits) << 16);
        }
        __syncthreads();
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // the second MMA of each step and token tile accumulates separately, so
    // consecutive MMAs do not wait on each other
    float acc[NT][4], accb[4] = {0.0f, 0.0f, 0.0f, 0.0f}, accc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float* acc2 = accb;                           // second MMA of token tile 0
    float* acc3 = NT > 1 ? accc : acc[NT - 1];    // second MMA of token tile 1
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;

    const __half* xrow0 = a.xp + (int64_t)g * a.ic + t * (F::kCols / 4);
    const __half* xrow1 = a.xp + (int64_t)(g + 8) * a.ic + t * (F::kCols / 4);
    const uint16_t* xb0 = static_cast<const uint16_t*>(a.x_raw) + (int64_t)g * a.ldx + t * (F::kCols / 4);
    const uint16_t* xb1 = static_cast<const uint16_t*>(a.x_raw) + (int64_t)(g + 8) * a.ldx + t * (F::kCols / 4);
    const bool tok0 = g < a.M, tok1 = (g + 8) < a.M;
    const int rg_first = u0 / nkc;
    const float* sig = BF ? nullptr : a.sigma;

    auto flush = [&](int rg, int seg0, int seg1) {
        if (seg0 == rg * nkc && seg1 == (rg + 1) * nkc) {
            write_rows<NT>(a, rg, acc, lane, sig);
            return;
        }
        const int slot = (rg == rg_first) ? 0 : 1;
        float* mine = a.partials + (((int64_t)gw * 2 + slot) * NT * 32 + lane) * 4;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            __stcg(reinterpret_cast<float4*>(mine + nt * 128), make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
        __syncwarp();
        const int64_t first = (int64_t)rg * nkc, last = (int64_t)(rg + 1) * nkc - 1;
        const int w_lo = (int)(((first + 1) * T - 1) / U), w_hi = (int)(((last + 1) * T - 1) / U);
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomic_add_acq_rel(a.counters + rg, 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != w_hi - w_lo) return;
        float sum[NT][4];
        const bool lo_second = (int)((int64_t)U * w_lo / T) / nkc != rg;
        sum_partials<NT>(a.partials, w_lo, w_hi, lo_second, lane, sum);
        write_rows<NT>(a, rg, sum, lane, sig);
        if (lane == 0) a.counters[rg] = 0;
    };

    int crg = rg_first, ckc = u0 - rg_first * nkc;
    int seg0 = u0;
    for (int i = 0; i < n; ++i) {
        const int st = i % kDepthT;
        cp_async_wait<kDepthT - 1>();
        uint32_t fw[FW];
        const uint4* slot = ring + st * (NV + 1) * 32;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const uint4 q = slot[v * 32];
            fw[4 * v] = q.x; fw[4 * v + 1] = q.y; fw[4 * v + 2] = q.z; fw[4 * v + 3] = q.w;
        }
        {
            const uint2 q = *reinterpret_cast<const uint2*>(slot + NV * 32);
            fw[4 * NV] = q.x; fw[4 * NV + 1] = q.y;
        }
        // the slot is reused by the copy issued next: consume the words first
#pragma unroll
        for (int k = 0; k < FW; ++k) asm volatile("" ::"r"(fw[k]));
        issue(u0 + i + kDepthT, st);
        if constexpr (FMT == SPARK_FMT_FP3) {
            // tiled FP3 code words back to the reference packing
            uint32_t ref[6];
            fp3_unpack_tiled(fw, ref);
#pragma unroll
            for (int k = 0; k < 6; ++k) fw[k] = ref[k];
            fp3_unpack_tiled(fw + 7, ref);
#pragma unroll
            for (int k = 0; k < 6; ++k) fw[7 + k] = ref[k];
        }

        const uint32_t* c0 = fw;
        const uint32_t* c1 = fw + FW / 2;
        uint32_t sw0 = 0, sw1 = 0;
        if constexpr (F::kScaleBytes != 0) { sw0 = fw[F::kChunkWords]; sw1 = fw[FW / 2 + F::kChunkWords]; }
        const int64_t col0 = (int64_t)ckc * F::kCols;
#pragma unroll
        for (int s = 0; s < F::kSteps; ++s) {
            uint32_t A0[4], A1[4];
            if constexpr (BF) {
                if constexpr (FMT == SPARK_FMT_SPFP2) {
                    decode_spfp2_bf16(c0, s, lut, A0);
                    decode_spfp2_bf16(c1, s, lut, A1);
                } else if constexpr (FMT == SPARK_FMT_TWOFOUR) {
                    decode_twofour_t<true>(c0, s, A0);
                    decode_twofour_t<true>(c1, s, A1);
                } else {
                    decode_scaled_bf16<FMT>(c0, sw0, s, pair_tab, scale_tab, A0);
                    decode_scaled_bf16<FMT>(c1, sw1, s, pair_tab, scale_tab, A1);
                }
                uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
                if (tok0) x0 = ldg_nc_v4(xb0 + col0 + 8 * s);
                if (NT > 1 && tok1) x1 = ldg_nc_v4(xb1 + col0 + 8 * s);
                mma_16816_bf16(acc[0], A0[0], A1[0], A0[1], A1[1], x0.x, x0.y);
                mma_16816_bf16(acc2, A0[2], A1[2], A0[3], A1[3], x0.z, x0.w);
                if (NT > 1) {
                    mma_16816_bf16(acc[NT - 1], A0[0], A1[0], A0[1], A1[1], x1.x, x1.y);
                    mma_16816_bf16(acc3, A0[2], A1[2], A0[3], A1[3], x1.z, x1.w);
                }
            } else {
                decode_step<FMT>(c0, sw0, s, A0);
                decode_step<FMT>(c1, sw1, s, A1);
#pragma unroll
                for (int part = 0; part < XS; ++part) {
                    const int64_t po = (int64_t)part * kMaxTokens * a.ic + col0 + 8 * s;
                    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
                    if (tok0) x0 = ldg_nc_v4(xrow0 + po);
                    if (NT > 1 && tok1) x1 = ldg_nc_v4(xrow1 + po);
                    mma_16816(acc[0], A0[0], A1[0], A0[1], A1[1], x0.x, x0.y);
                    mma_16816(acc2, A0[2], A1[2], A0[3], A1[3], x0.z, x0.w);
                    if (NT > 1) {
                        mma_16816(acc[NT - 1], A0[0], A1[0], A0[1], A1[1], x1.x, x1.y);
                        mma_16816(acc3, A0[2], A1[2], A0[3], A1[3], x1.z, x1.w);
                    }
                }
            }
        }
        const int u = u0 + i;
        if (++ckc == nkc || i + 1 == n) {
#pragma unroll
            for (int q = 0; q < 4; ++q) { acc[0][q] += accb[q]; accb[q] = 0.0f; }
            if constexpr (NT > 1) {
#pragma unroll
                for (int q = 0; q < 4; ++q) { acc[NT - 1][q] += accc[q]; accc[q] = 0.0f; }
            }
            flush(crg, seg0, u + 1);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[nt][q] = 0.0f;
            if (ckc == nkc) { ckc = 0; ++crg; }
            seg0 = u + 1;
        }
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------- generic path
// Any shape / alignment / format, one warp per output row: decode from global
// memory with byte loads and accumulate in fp32.  Used when the fast path's
// layout conditions do not hold (small or ragged layers, the v1 format).
__device__ __forceinline__ float decode_generic(int fmt, const uint8_t* wq, const uint8_t* sc, int64_t ic,
                                                int64_t r, int64_t c) {
    if (fmt == SPARK_FMT_SPFP2 || fmt == SPARK_FMT_SPFP2_V1) {
        // flattened block index over the row-major weight (pairs may straddle rows)
        const int64_t k = r * ic + c;
        const int64_t b = k >> 3;
        const int i = (int)(k & 7);
        uint32_t m, e;
        if (fmt == SPARK_FMT_SPFP2) {
            const uint8_t* q = wq + (b >> 1) * 5;
            const int h = (int)(b & 1);
            m = (uint32_t)q[2 * h] | ((uint32_t)q[2 * h + 1] << 8);
            e = h ? (q[4] >> 4) : (q[4] & 0xfu);
        } else {
            const uint8_t* q = wq + b * 3;
            m = (uint32_t)q[0] | ((uint32_t)q[1] << 8);
            e = q[2] & 0xfu;
        }
        const uint32_t code = (m >> (2 * i)) & 3u;
        const float s = spfp2_scale((int)e);
        return code == 0 ? s : (code == 1 ? -s : 0.0f);
    }
    const int64_t nbr = (ic + 15) / 16;
    const int64_t k = (r * nbr) * 16 + c;        // row-padded code index
    if (fmt == SPARK_FMT_FP3) {
        const int64_t gi = k >> 3;
        const uint8_t* q = wq + gi * 3;
        const uint32_t v = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16);
        const uint32_t code = (v >> (3 * (k & 7))) & 7u;
        const float tbl[8] = {0.0f, 0.5f, 1.0f, 1.5f, -0.0f, -0.5f, -1.0f, -1.5f};
        return tbl[code] * e4m3_to_f32(sc[k >> 4]);
    }
    if (fmt == SPARK_FMT_NVFP4) {
        const uint32_t byte = wq[k >> 1];
        const uint32_t code = (k & 1) ? (byte >> 4) : (byte & 0xfu);
        const float pos[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
        const float v = code < 8 ? pos[code] : -pos[code - 8];
        return v * e4m3_to_f32(sc[k >> 4]);
    }
    // 2:4: blocks of 16 over the row-padded flattening, pairs of blocks in 7 bytes
    const int64_t b = k >> 4;
    const int pos = (int)(k & 15);
    const uint8_t* q = wq + (b >> 1) * 7;
    uint64_t v = 0;
    for (int i = 0; i < 7; ++i) v |= (uint64_t)q[i] << (8 * i);
    const uint32_t w = (uint32_t)(v >> (28 * (b & 1))) & 0x0fffffffu;
    const float s = spfp2_scale((int)((w >> 24) & 0xfu));
    const int grp = pos >> 2, p = pos & 3;
    const uint32_t mode = (w >> (4 * grp)) & 0xfu;
    const float n0 = ((w >> (16 + 2 * grp)) & 1u) ? -s : s;
    const float n1 = ((w >> (17 + 2 * grp)) & 1u) ? -s : s;
    if (mode < 6u) {
        const int pa = mode < 3u ? 0 : (mode < 5u ? 1 : 2);
        const int pb = mode == 0u ? 1 : (mode == 1u ? 2 : ((mode == 2u || mode == 4u || mode == 5u) ? 3 : 2));
        return p == pa ? n0 : (p == pb ? n1 : 0.0f);
    }
    if (mode >= 8u && mode <= 11u) return p == (int)mode - 8 ? n0 : 0.0f;
    return 0.0f;
}

__global__ void __launch_bounds__(256) k_linear_generic(int fmt, const uint8_t* __restrict__ wq,
                                                        const uint8_t* __restrict__ sc, const void* __restrict__ x,
                                                        int x_dtype, int64_t M, int64_t oc, int64_t ic, int64_t ldx,
                                                        const void* __restrict__ bias, int bias_dtype,
                                                        void* __restrict__ y, int y_dtype, int64_t ldy) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= oc) return;
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t c = lane; c < ic; c += 32) {
            const float w = decode_generic(fmt, wq, sc, ic, r, c);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (m0 + j < M) acc[j] += w * load_as_float(x, x_dtype, (m0 + j) * ldx + c);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float v = acc[j];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && m0 + j < M) {
                if (bias) v += load_as_float(bias, bias_dtype, r);
                store_from_float(y, y_dtype, (m0 + j) * ldy + r, v);
            }
        }
    }
}

// ---------------------------------------------------------------- host side
struct DeviceInfo {
    int sms = 0;
    bool attrs_set[8] = {};
};
DeviceInfo g_dev[64];
std::mutex g_mu;

int sm_count(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_dev[dev].sms == 0) cudaDeviceGetAttribute(&g_dev[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    return g_dev[dev].sms;
}

template <int FMT>
size_t gemv_smem() {
    return (size_t)kWarps * kDepth * stage_bytes<FMT>() + (size_t)kWarps * kDepth * 8;
}

template <int FMT, int NT, int XS>
int set_smem_attr(int dev) {
    static bool done[64] = {};
    std::lock_guard<std::mutex> lk(g_mu);
    if (!done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<FMT, NT, XS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)gemv_smem<FMT>());
        if (e != cudaSuccess) return set_error((int)e, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        done[dev] = true;
    }
    return SPARK_OK;
}

int cols_per_unit(int fmt) { return fmt == SPARK_FMT_TWOFOUR ? 512 : 256; }

// Workspace layout (bytes).  Everything whose contents must survive from one
// call to the next (the self-resetting row-group counters) sits at an offset
// that does not depend on the problem shape; only the prepared activations,
// which every call rewrites, grow with ic.
constexpr int64_t kMaxRowGroups = 1 << 16;   // oc <= 1,048,576
struct WsLayout {
    size_t err = 0;                            // int error word
    // [64, 4096): control block of the batched decode kernel (stream.cu)
    size_t sigma = 4096;                       // float[16]
    size_t counters = 4352;                    // int[kMaxRowGroups]
    size_t partials = 0;                       // float[T][2][2*32*4]
    size_t xp = 0;                             // half[2][16][ic] (hi, lo parts)
    size_t total = 0;
};

WsLayout ws_layout(int64_t ic, int64_t T) {
    WsLayout L;
    L.partials = L.counters + (size_t)kMaxRowGroups * sizeof(int);
    L.xp = L.partials + (size_t)T * 2 * 2 * 32 * 4 * sizeof(float);
    L.total = (L.xp + (size_t)2 * kMaxTokens * ic * 2 + 255) / 256 * 256;
    return L;
}

int64_t max_warps(int dev) { return (int64_t)sm_count(dev) * 2 * kWarps; }

template <int FMT, int NT, int XS>
int launch_gemv(const GemvArgs& a, int64_t T, cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    int rc = set_smem_attr<FMT, NT, XS>(dev);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(T / kWarps));
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = gemv_smem<FMT>();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv<FMT, NT, XS>, a);
    if (e != cudaSuccess) return set_error((int)e, "k_gemv launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

template <int FMT>
int launch_fmt(const GemvArgs& a, int NT, int XS, int64_t T, cudaStream_t s) {
    if (XS == 1) return NT == 1 ? launch_gemv<FMT, 1, 1>(a, T, s) : launch_gemv<FMT, 2, 1>(a, T, s);
    return NT == 1 ? launch_gemv<FMT, 1, 2>(a, T, s) : launch_gemv<FMT, 2, 2>(a, T, s);
}

template <int FMT>
size_t gemv_tiled_smem() {
    return (size_t)kWarps * kDepthT * (frag_words<FMT>() / 4 + 1) * 32 * 16;
}

template <int FMT, int NT, int XS, bool BF>
int launch_gemv_tiled(const GemvArgs& a, int64_t T, cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = gemv_tiled_smem<FMT>();
    {
        static bool done[64] = {};
        std::lock_guard<std::mutex> lk(g_mu);
        if (!done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(k_gemv_tiled<FMT, NT, XS, BF>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return set_error((int)e, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(T / kWarps));
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_tiled<FMT, NT, XS, BF>, a);
    if (e != cudaSuccess) return set_error((int)e, "k_gemv_tiled launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

template <int FMT>
int launch_fmt_tiled(const GemvArgs& a, int NT, int XS, bool bf, int64_t T, cudaStream_t s) {
    if (bf) return NT == 1 ? launch_gemv_tiled<FMT, 1, 1, true>(a, T, s) : launch_gemv_tiled<FMT, 2, 1, true>(a, T, s);
    if (XS == 1) return NT == 1 ? launch_gemv_tiled<FMT, 1, 1, false>(a, T, s) : launch_gemv_tiled<FMT, 2, 1, false>(a, T, s);
    return NT == 1 ? launch_gemv_tiled<FMT, 1, 2, false>(a, T, s) : launch_gemv_tiled<FMT, 2, 2, false>(a, T, s);
}

int launch_prepare(const void* x, int x_dtype, int64_t ldx, int64_t ic, int fmt, __half* xp, float* sigma, int split,
                   int mc, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)mc);
    cfg.blockDim = dim3(kPrepThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_prepare_x, x, x_dtype, ldx, ic, fmt, xp, sigma, split);
    if (e != cudaSuccess) return set_error((int)e, "k_prepare_x launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

int64_t tiled_bytes(int fmt, int64_t oc, int64_t ic) {
    if (fmt != SPARK_FMT_SPFP2 && fmt != SPARK_FMT_FP3 && fmt != SPARK_FMT_NVFP4 && fmt != SPARK_FMT_TWOFOUR) return 0;
    if (oc <= 0 || ic <= 0 || ic % cols_per_unit(fmt) != 0) return 0;
    const int64_t units = (oc + 15) / 16 * (ic / cols_per_unit(fmt));
    if (units < kWarps) return 0;
    int ub = 0;
    switch (fmt) {
        case SPARK_FMT_SPFP2: ub = unit_bytes_tiled<SPARK_FMT_SPFP2>(); break;
        case SPARK_FMT_FP3: ub = unit_bytes_tiled<SPARK_FMT_FP3>(); break;
        case SPARK_FMT_NVFP4: ub = unit_bytes_tiled<SPARK_FMT_NVFP4>(); break;
        default: ub = unit_bytes_tiled<SPARK_FMT_TWOFOUR>(); break;
    }
    return units * ub;
}

bool fast_path_ok(int fmt, const uint8_t* wq, const uint8_t* scales, int64_t oc, int64_t ic) {
    if (fmt == SPARK_FMT_SPFP2_V1) return false;
    if (ic % cols_per_unit(fmt) != 0) return false;
    if (!aligned(wq, 16)) return false;
    if ((fmt == SPARK_FMT_FP3 || fmt == SPARK_FMT_NVFP4) && !aligned(scales, 16)) return false;
    const int64_t units = (oc + 15) / 16 * (ic / cols_per_unit(fmt));
    return units >= kWarps;
}

}  // namespace

}  // namespace spark

namespace spark {
struct StreamPlan;
int stream_plan_alloc(StreamPlan** P);
void stream_plan_free(StreamPlan* P);
size_t stream_plan_scratch(const StreamPlan* P);
int stream_plan(const SparkChainOp* ops, int n_ops, int64_t M, uint8_t* ws, size_t counters_off,
                int64_t max_counters, size_t scratch_off, StreamPlan* P);
int stream_launch(const StreamPlan& P, cudaStream_t s);
int stream_plan_set_ar(StreamPlan* P, const SparkBatchAllReduce* ar);
int twofour_sparse_run(const uint8_t* wq, const void* x, int64_t M, int64_t oc, int64_t ic, const void* bias,
                       int bias_dtype, void* y, int y_dtype, int64_t ldy, int* err, int* counters, float* part,
                       size_t part_bytes, cudaStream_t stream);
constexpr int64_t kSplitMaxTok = 16;    // 2:4 token counts whose sparse launch splits K
size_t stream_scratch_single(int64_t M, int64_t ic);
size_t tc_partials_bytes(int dev, int64_t M);
bool tc_linear_ok(int fmt, const void* wq, const void* scales, const void* x, int x_dtype, int64_t ic,
                  int64_t ldx);
int tc_linear(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int64_t M, int64_t oc, int64_t ic,
              int64_t ldx, const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy, int* err,
              int* counters, int64_t max_counters, float* partials, cudaStream_t s);
}  // namespace spark

// ====================================================================== C ABI
using namespace spark;

extern "C" {

size_t spark_linear_workspace_size(int fmt, int64_t M, int64_t oc, int64_t ic) {
    (void)fmt;
    (void)oc;
    int dev = 0;
    cudaGetDevice(&dev);
    const WsLayout L = ws_layout(ic, max_warps(dev));
    return std::max({L.total, L.partials + tc_partials_bytes(dev, M), L.partials + stream_scratch_single(M, ic)});
}

int spark_linear(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype, int64_t M,
                 int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype, void* y, int y_dtype,
                 int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
    return spark_linear_prefetch(fmt, wq, scales, x, x_dtype, M, oc, ic, ldx, bias, bias_dtype, y, y_dtype, ldy,
                                 workspace, workspace_bytes, nullptr, 0, stream);
}

int spark_linear_prefetch(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype, int64_t M,
                          int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype, void* y, int y_dtype,
                          int64_t ldy, void* workspace, size_t workspace_bytes, const void* prefetch,
                          int64_t prefetch_bytes, void* stream) {
    SPARK_REQUIRE(prefetch_bytes >= 0 && (!prefetch || aligned(prefetch, 16)), SPARK_ERR_ALIGNMENT,
                  "spark_linear_prefetch: the prefetch range must start on 16 bytes");
    const bool tiled = (fmt & SPARK_LAYOUT_TILED) != 0;
    const bool tcgen05 = (fmt & SPARK_PATH_TCGEN05) != 0;
    const bool silu = (fmt & SPARK_EPILOGUE_SILU) != 0;
    fmt &= ~(SPARK_LAYOUT_TILED | SPARK_PATH_TCGEN05 | SPARK_EPILOGUE_SILU);
    SPARK_REQUIRE(fmt >= SPARK_FMT_SPFP2 && fmt <= SPARK_FMT_TWOFOUR, SPARK_ERR_INVALID, "spark_linear: bad format %d", fmt);
    SPARK_REQUIRE(!tiled || tiled_bytes(fmt, oc, ic) > 0, SPARK_ERR_INVALID,
                  "spark_linear: no tiled layout for format %d [%lld, %lld]", fmt, (long long)oc, (long long)ic);
    SPARK_REQUIRE(wq && x && y, SPARK_ERR_INVALID, "spark_linear: null pointer");
    SPARK_REQUIRE(M >= 0 && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_linear: negative size");
    SPARK_REQUIRE(ldx >= ic && ldy >= (silu ? oc / 2 : oc), SPARK_ERR_INVALID,
                  "spark_linear: ldx %lld < ic or ldy %lld below the output width", (long long)ldx, (long long)ldy);
    SPARK_REQUIRE(!silu || oc % 16 == 0, SPARK_ERR_INVALID,
                  "spark_linear: the fused SiLU epilogue takes whole 16-row groups (8 gate + 8 up rows)");
    SPARK_REQUIRE(tiled || (fmt != SPARK_FMT_FP3 && fmt != SPARK_FMT_NVFP4) || scales, SPARK_ERR_INVALID,
                  "spark_linear: FP3/NVFP4 need scales");
    SPARK_REQUIRE(x_dtype >= 0 && x_dtype <= 2 && y_dtype >= 0 && y_dtype <= 2 && bias_dtype >= 0 && bias_dtype <= 2,
                  SPARK_ERR_INVALID, "spark_linear: bad dtype");
    if (M == 0 || oc == 0) return SPARK_OK;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // More than 16 tokens on a reference layout with bf16 x: the tcgen05 GEMM.
    const bool tc_ok = !tiled && tc_linear_ok(fmt, wq, scales, x, x_dtype, ic, ldx);
    // 2:4 weights: the tcgen05 kernel at every token count (its decode GEMV is far slower)
    if (tcgen05 || (tc_ok && (M > kMaxTokens || fmt == SPARK_FMT_TWOFOUR))) {
        SPARK_REQUIRE(!silu, SPARK_ERR_UNSUPPORTED,
                      "spark_linear: the fused SiLU epilogue runs on the decode GEMV (tiled weights, or up to 16 "
                      "tokens on the reference layout)");
        SPARK_REQUIRE(tc_ok, SPARK_ERR_UNSUPPORTED,
                      "spark_linear: the tcgen05 path takes SPFP2, FP3 or NVFP4 in the reference layout, bf16 x, "
                      "ic %% 256 == 0, 16-byte aligned weights, scales and x, ldx %% 8 == 0");
        int dev = 0;
        cudaGetDevice(&dev);
        const WsLayout L = ws_layout(ic, max_warps(dev));
        const size_t need = L.partials + tc_partials_bytes(dev, M);
        SPARK_REQUIRE(workspace && workspace_bytes >= need, SPARK_ERR_WORKSPACE,
                      "spark_linear: workspace of %zu bytes needed (got %zu)", need, workspace_bytes);
        SPARK_REQUIRE(aligned(workspace, 256), SPARK_ERR_ALIGNMENT, "spark_linear: workspace must be 256-byte aligned");
        uint8_t* ws = static_cast<uint8_t*>(workspace);
        // 2:4 at up to 16 tokens and at 128 to 1024: the sparse tensor-core
        // kernel, which keeps the two nonzeros of every group and skips the
        // zero half of the MMA.  Up to 16 tokens it splits K over the SMs (the
        // partial sums in the workspace's partial area): down_proj 2560x9728
        // 21 -> 15 us at one token; at 128-1024 tokens 71-73 -> 53-55 us.  In
        // between (32-64 tokens) the dense decode measured faster.
        const bool sparse_small = M <= kSplitMaxTok, sparse_mid = M >= 128 && M <= 1024;
        if (fmt == SPARK_FMT_TWOFOUR && !tcgen05 && (sparse_small || sparse_mid) && oc % 128 == 0 &&
            ic % 128 == 0 && ldx == ic && aligned(wq, 4))
            return twofour_sparse_run(wq, x, M, oc, ic, bias, bias_dtype, y, y_dtype, ldy,
                                      reinterpret_cast<int*>(ws + L.err),
                                      sparse_small ? reinterpret_cast<int*>(ws + L.counters) : nullptr,
                                      sparse_small ? reinterpret_cast<float*>(ws + L.partials) : nullptr,
                                      tc_partials_bytes(dev, M), s);
        return tc_linear(fmt, wq, scales, x, M, oc, ic, ldx, bias, bias_dtype, y, y_dtype, ldy,
                               reinterpret_cast<int*>(ws + L.err), reinterpret_cast<int*>(ws + L.counters),
                               kMaxRowGroups, reinterpret_cast<float*>(ws + L.partials), s);
    }
    if (tiled && fmt != SPARK_FMT_TWOFOUR && x_dtype == SPARK_DTYPE_BF16 && aligned(x, 16) && ldx % 8 == 0) {
        // bf16 activations on tiled SPFP2 / FP3 / NVFP4: the batched decode
        // kernel (stream.cu), one op per 16-token chunk
        int dev = 0;
        cudaGetDevice(&dev);
        const WsLayout L = ws_layout(ic, max_warps(dev));
        SPARK_REQUIRE(workspace && aligned(workspace, 256), SPARK_ERR_WORKSPACE,
                      "spark_linear: a 256-byte aligned workspace is required");
        StreamPlan* P = nullptr;
        int rc = stream_plan_alloc(&P);
        if (rc) return rc;
        for (int64_t m0 = 0; m0 < M && rc == SPARK_OK; m0 += kMaxTokens) {
            const int64_t mc = std::min<int64_t>(kMaxTokens, M - m0);
            SparkChainOp op = {};
            op.kind = SPARK_CHAIN_LINEAR;
            op.fmt = fmt | SPARK_LAYOUT_TILED | (silu ? SPARK_EPILOGUE_SILU : 0);
            op.wq = wq;
            op.x = static_cast<const uint16_t*>(x) + m0 * ldx;
            op.ic = ic;
            op.ldx = ldx;
            op.oc = oc;
            op.bias = bias;
            op.bias_dtype = bias_dtype;
            op.y = static_cast<uint8_t*>(y) + m0 * ldy * (y_dtype == SPARK_DTYPE_F32 ? 4 : 2);
            op.y_dtype = y_dtype;
            op.ldy = ldy;
            op.dep[0] = op.dep[1] = -1;
            rc = stream_plan(&op, 1, mc, static_cast<uint8_t*>(workspace), L.counters, kMaxRowGroups, L.partials, P);
            if (rc == SPARK_OK && L.partials + stream_plan_scratch(P) > workspace_bytes)
                rc = set_error(SPARK_ERR_WORKSPACE, "spark_linear: workspace of %zu bytes needed (got %zu)",
                               L.partials + stream_plan_scratch(P), workspace_bytes);
            if (rc == SPARK_OK) rc = stream_launch(*P, s);
        }
        stream_plan_free(P);
        return rc;
    }
    SPARK_REQUIRE(!(tiled && fmt == SPARK_FMT_SPFP2), SPARK_ERR_UNSUPPORTED,
                  "spark_linear: tiled SPFP2 weights take bf16 activations (16-byte aligned, ldx %% 8 == 0); "
                  "use the reference layout for other activations");
    if (tiled) {
        SPARK_REQUIRE(aligned(wq, 16), SPARK_ERR_ALIGNMENT, "spark_linear: tiled weights must be 16-byte aligned");
    } else if (!fast_path_ok(fmt, wq, scales, oc, ic)) {
        SPARK_REQUIRE(!silu, SPARK_ERR_UNSUPPORTED, "spark_linear: no fused SiLU epilogue for this shape / alignment");
        k_linear_generic<<<(unsigned)((oc + 7) / 8), 256, 0, s>>>(fmt, wq, scales, x, x_dtype, M, oc, ic, ldx, bias,
                                                                  bias_dtype, y, y_dtype, ldy);
        return check_launch("spark_linear (generic)");
    }
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t Tmax = max_warps(dev);
    const WsLayout L = ws_layout(ic, Tmax);
    SPARK_REQUIRE(workspace && workspace_bytes >= L.total, SPARK_ERR_WORKSPACE,
                  "spark_linear: workspace of %zu bytes needed (got %zu)", L.total, workspace_bytes);
    SPARK_REQUIRE(aligned(workspace, 256), SPARK_ERR_ALIGNMENT, "spark_linear: workspace must be 256-byte aligned");
    SPARK_REQUIRE((oc + 15) / 16 <= kMaxRowGroups, SPARK_ERR_UNSUPPORTED, "spark_linear: oc %lld above %lld",
                  (long long)oc, (long long)(16 * kMaxRowGroups));

    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int64_t units = (oc + 15) / 16 * (ic / cols_per_unit(fmt));
    SPARK_REQUIRE(units < (1ll << 30), SPARK_ERR_UNSUPPORTED, "spark_linear: layer too large for one launch");
    int64_t T = std::min(Tmax, units) / kWarps * kWarps;
    GemvArgs a = {};
    a.wq = wq;
    a.scales = scales;
    a.xp = reinterpret_cast<const __half*>(ws + L.xp);
    a.sigma = reinterpret_cast<const float*>(ws + L.sigma);
    a.bias = bias;
    a.partials = reinterpret_cast<float*>(ws + L.partials);
    a.counters = reinterpret_cast<int*>(ws + L.counters);
    a.err = reinterpret_cast<int*>(ws + L.err);
    a.oc = oc;
    a.ic = ic;
    a.ldy = ldy;
    a.bias_dtype = bias_dtype;
    a.y_dtype = y_dtype;
    a.n_rg = (oc + 15) / 16;
    a.n_kc = ic / cols_per_unit(fmt);
    a.units = units;
    switch (fmt) {
        case SPARK_FMT_SPFP2: a.row_bytes = Fmt<SPARK_FMT_SPFP2>::row_bytes(ic); break;
        case SPARK_FMT_FP3: a.row_bytes = Fmt<SPARK_FMT_FP3>::row_bytes(ic); break;
        case SPARK_FMT_NVFP4: a.row_bytes = Fmt<SPARK_FMT_NVFP4>::row_bytes(ic); break;
        default: a.row_bytes = Fmt<SPARK_FMT_TWOFOUR>::row_bytes(ic); break;
    }
    a.scale_row_bytes = ic / 16;
    a.silu_pairs = silu ? 1 : 0;
    a.pf = static_cast<const uint8_t*>(prefetch);
    a.pf_bytes = prefetch ? prefetch_bytes / 16 * 16 : 0;

    for (int64_t m0 = 0; m0 < M; m0 += kMaxTokens) {
        const int mc = (int)std::min<int64_t>(kMaxTokens, M - m0);
        const uint8_t* xb = static_cast<const uint8_t*>(x) + m0 * ldx * (x_dtype == SPARK_DTYPE_F32 ? 4 : 2);
        const int XS = x_dtype == SPARK_DTYPE_BF16 ? 1 : 2;
        // tiled weights with bf16 x: bf16 MMA straight on x, no prepare launch
        const bool bf = tiled && x_dtype == SPARK_DTYPE_BF16 && (ldx % 8) == 0 && aligned(x, 16);
        a.x_raw = xb;
        a.ldx = ldx;
        const int perm = fmt == SPARK_FMT_FP3 ? kPermFp3 : (fmt == SPARK_FMT_SPFP2 && !tiled ? kPermSpfp2 : kPermNatural);
        int rc = SPARK_OK;
        if (!bf) rc = launch_prepare(xb, x_dtype, ldx, ic, perm, reinterpret_cast<__half*>(ws + L.xp),
                                reinterpret_cast<float*>(ws + L.sigma), XS == 2, mc, s);
        if (rc) return rc;
        a.M = mc;
        a.y = static_cast<uint8_t*>(y) + m0 * ldy * (y_dtype == SPARK_DTYPE_F32 ? 4 : 2);
        const int NT = mc > 8 ? 2 : 1;
        if (tiled) {
            switch (fmt) {
                case SPARK_FMT_FP3: rc = launch_fmt_tiled<SPARK_FMT_FP3>(a, NT, XS, bf, T, s); break;
                case SPARK_FMT_NVFP4: rc = launch_fmt_tiled<SPARK_FMT_NVFP4>(a, NT, XS, bf, T, s); break;
                default: rc = launch_fmt_tiled<SPARK_FMT_TWOFOUR>(a, NT, XS, bf, T, s); break;
            }
            if (rc) return rc;
            continue;
        }
        switch (fmt) {
            case SPARK_FMT_SPFP2: rc = launch_fmt<SPARK_FMT_SPFP2>(a, NT, XS, T, s); break;
            case SPARK_FMT_FP3: rc = launch_fmt<SPARK_FMT_FP3>(a, NT, XS, T, s); break;
            case SPARK_FMT_NVFP4: rc = launch_fmt<SPARK_FMT_NVFP4>(a, NT, XS, T, s); break;
            default: rc = launch_fmt<SPARK_FMT_TWOFOUR>(a, NT, XS, T, s); break;
        }
        if (rc) return rc;
    }
    return SPARK_OK;
}

size_t spark_tiled_bytes(int fmt, int64_t oc, int64_t ic) { return (size_t)tiled_bytes(fmt, oc, ic); }

int spark_tile_weights(int fmt, const uint8_t* wq, const uint8_t* scales, int64_t oc, int64_t ic, uint8_t* tiled,
                       void* stream) {
    SPARK_REQUIRE(wq && tiled, SPARK_ERR_INVALID, "spark_tile_weights: null pointer");
    SPARK_REQUIRE(tiled_bytes(fmt, oc, ic) > 0, SPARK_ERR_UNSUPPORTED,
                  "spark_tile_weights: format %d [%lld, %lld] has no tiled layout (ic %% %d != 0 or too small)", fmt,
                  (long long)oc, (long long)ic, fmt == SPARK_FMT_TWOFOUR ? 512 : 256);
    SPARK_REQUIRE((fmt != SPARK_FMT_FP3 && fmt != SPARK_FMT_NVFP4) || scales, SPARK_ERR_INVALID,
                  "spark_tile_weights: FP3/NVFP4 need scales");
    SPARK_REQUIRE(aligned(wq, 16) && aligned(tiled, 16) && (!scales || aligned(scales, 4)), SPARK_ERR_ALIGNMENT,
                  "spark_tile_weights: buffers must be 16-byte aligned");
    const int64_t n_kc = ic / cols_per_unit(fmt);
    const int64_t units = (oc + 15) / 16 * n_kc;
    const unsigned grid = (unsigned)((units * 32 + 255) / 256);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (fmt) {
        case SPARK_FMT_SPFP2:
            k_tile<SPARK_FMT_SPFP2><<<grid, 256, 0, s>>>(wq, scales, oc, Fmt<SPARK_FMT_SPFP2>::row_bytes(ic), ic / 16,
                                                          n_kc, units, tiled);
            break;
        case SPARK_FMT_FP3:
            k_tile<SPARK_FMT_FP3><<<grid, 256, 0, s>>>(wq, scales, oc, Fmt<SPARK_FMT_FP3>::row_bytes(ic), ic / 16, n_kc,
                                                        units, tiled);
            break;
        case SPARK_FMT_NVFP4:
            k_tile<SPARK_FMT_NVFP4><<<grid, 256, 0, s>>>(wq, scales, oc, Fmt<SPARK_FMT_NVFP4>::row_bytes(ic), ic / 16,
                                                          n_kc, units, tiled);
            break;
        default:
            k_tile<SPARK_FMT_TWOFOUR><<<grid, 256, 0, s>>>(wq, scales, oc, Fmt<SPARK_FMT_TWOFOUR>::row_bytes(ic),
                                                            ic / 16, n_kc, units, tiled);
            break;
    }
    return check_launch("spark_tile_weights");
}

size_t spark_linear_batch_workspace_size(const SparkChainOp* ops, int n_ops, int64_t M) {
    int dev = 0;
    cudaGetDevice(&dev);
    const WsLayout L = ws_layout(0, max_warps(dev));
    StreamPlan* P = nullptr;
    if (stream_plan_alloc(&P)) return 0;
    size_t need = 0;
    if (stream_plan(ops, n_ops, M, nullptr, L.counters, kMaxRowGroups, L.partials, P) == SPARK_OK)
        need = (L.partials + stream_plan_scratch(P) + 255) / 256 * 256;
    stream_plan_free(P);
    return need;
}

int spark_linear_batch(const SparkChainOp* ops, int n_ops, int64_t M, void* workspace, size_t workspace_bytes,
                       void* stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    const WsLayout L = ws_layout(0, max_warps(dev));
    SPARK_REQUIRE(workspace && aligned(workspace, 256), SPARK_ERR_WORKSPACE,
                  "spark_linear_batch: a 256-byte aligned workspace is required");
    StreamPlan* P = nullptr;
    int rc = stream_plan_alloc(&P);
    if (rc) return rc;
    rc = stream_plan(ops, n_ops, M, static_cast<uint8_t*>(workspace), L.counters, kMaxRowGroups, L.partials, P);
    if (rc == SPARK_OK && L.partials + stream_plan_scratch(P) > workspace_bytes)
        rc = set_error(SPARK_ERR_WORKSPACE, "spark_linear_batch: workspace of %zu bytes needed (got %zu)",
                       L.partials + stream_plan_scratch(P), workspace_bytes);
    if (rc == SPARK_OK) rc = stream_launch(*P, reinterpret_cast<cudaStream_t>(stream));
    stream_plan_free(P);
    return rc;
}

int64_t spark_batch_ar_recv_bytes(int world, int64_t M, int64_t oc) {
    if (world < 1 || world > SPARK_MAX_PEERS || M < 1 || M > 16 || oc < 1) return 0;
    return (int64_t)2 * world * ((oc + 15) / 16) * M * 16 * 8;
}

}  // extern "C"

// The host-side checks of the all-reduce arguments that need no device.
static int check_batch_ar(const SparkChainOp* ops, int n_ops, const SparkBatchAllReduce* ar) {
    SPARK_REQUIRE(ar, SPARK_ERR_INVALID, "spark_linear_batch_ar: null all-reduce arguments");
    SPARK_REQUIRE(ar->world >= 1 && ar->world <= SPARK_MAX_PEERS && ar->rank >= 0 && ar->rank < ar->world,
                  SPARK_ERR_INVALID, "spark_linear_batch_ar: rank %d of %d (1 to %d ranks)", ar->rank, ar->world,
                  SPARK_MAX_PEERS);
    SPARK_REQUIRE(ops && ar->op >= 0 && ar->op < n_ops, SPARK_ERR_INVALID,
                  "spark_linear_batch_ar: op %d not in the batch", ar->op);
    // the summed output is written after the op's units complete, so no op
    // of the same launch can wait for it
    for (int k = 0; k < n_ops; ++k)
        SPARK_REQUIRE(ops[k].dep[0] != ar->op && ops[k].dep[1] != ar->op, SPARK_ERR_UNSUPPORTED,
                      "spark_linear_batch_ar: op %d reads the all-reduced op %d; run it in a later launch", k,
                      ar->op);
    return SPARK_OK;
}

extern "C" {

size_t spark_linear_batch_ar_workspace_size(const SparkChainOp* ops, int n_ops, int64_t M,
                                            const SparkBatchAllReduce* ar) {
    if (check_batch_ar(ops, n_ops, ar) != SPARK_OK) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const WsLayout L = ws_layout(0, max_warps(dev));
    StreamPlan* P = nullptr;
    if (stream_plan_alloc(&P)) return 0;
    size_t need = 0;
    if (stream_plan(ops, n_ops, M, nullptr, L.counters, kMaxRowGroups, L.partials, P) == SPARK_OK &&
        stream_plan_set_ar(P, ar) == SPARK_OK)
        need = (L.partials + stream_plan_scratch(P) + 255) / 256 * 256;
    stream_plan_free(P);
    return need;
}

int spark_linear_batch_ar(const SparkChainOp* ops, int n_ops, int64_t M, const SparkBatchAllReduce* ar,
                          void* workspace, size_t workspace_bytes, void* stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    const WsLayout L = ws_layout(0, max_warps(dev));
    SPARK_REQUIRE(workspace && aligned(workspace, 256), SPARK_ERR_WORKSPACE,
                  "spark_linear_batch_ar: a 256-byte aligned workspace is required");
    int rc = check_batch_ar(ops, n_ops, ar);
    if (rc) return rc;
    StreamPlan* P = nullptr;
    rc = stream_plan_alloc(&P);
    if (rc) return rc;
    rc = stream_plan(ops, n_ops, M, static_cast<uint8_t*>(workspace), L.counters, kMaxRowGroups, L.partials, P);
    if (rc == SPARK_OK) rc = stream_plan_set_ar(P, ar);
    if (rc == SPARK_OK && L.partials + stream_plan_scratch(P) > workspace_bytes)
        rc = set_error(SPARK_ERR_WORKSPACE, "spark_linear_batch_ar: workspace of %zu bytes needed (got %zu)",
                       L.partials + stream_plan_scratch(P), workspace_bytes);
    if (rc == SPARK_OK) rc = stream_launch(*P, reinterpret_cast<cudaStream_t>(stream));
    stream_plan_free(P);
    return rc;
}

int spark_workspace_check(void* workspace, void* stream) {
    SPARK_REQUIRE(workspace, SPARK_ERR_INVALID, "spark_workspace_check: null workspace");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int flag = 0;
    cudaError_t e = cudaMemcpyAsync(&flag, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return set_error((int)e, "spark_workspace_check: %s", cudaGetErrorString(e));
    if (flag != 0) {
        cudaMemsetAsync(workspace, 0, sizeof(int), s);
        return set_error(SPARK_ERR_DEVICE, "a kernel reported error %d (%s)", flag,
                         flag == 7 ? "embedding id out of range" : "bounded wait expired");
    }
    return SPARK_OK;
}

}  // extern "C"

// ====================================================================== no-allocation entry point
// Some callers may not allocate device memory when they run a linear: an
// inference runtime whose memory plan is fixed before the first token, a host
// that hands its whole budget to a caching allocator it cannot re-enter from
// the decode loop, or a C caller with no allocator at all.  Both kernels
// behind spark_linear still need scratch: the decode GEMV its error word,
// row-group counters, split partials, per-token scales and prepared
// activations; the tcgen05 GEMM its error word, job counters and stream-K
// partials.  spark_linear_noalloc takes that scratch from one statically sized
// array in this module (one copy per device) instead of a caller-provided
// workspace, and allocates nothing.  16 MiB covers the tcgen05 route at any
// token count (266,496 + 2 * SMs * 64 * 128 * 4 bytes: 9.97 MB on 148 SMs) and
// the decode GEMV up to ic = 182,204 on 148 SMs.
namespace spark {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of this device's scratch.  The first call on a device looks
// the symbol up with that device current and clears the part whose contents
// must start at zero: the error word and the row-group counters (the kernels
// return the counters to zero themselves; everything after them is written
// before it is read).  The clear is synchronised so that later calls on any
// stream see it.
int noalloc_scratch(int dev, cudaStream_t s, void** out) {
    SPARK_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, SPARK_ERR_UNSUPPORTED,
                  "spark_linear_noalloc: device ordinal %d above %d", dev, kNoAllocMaxDevices - 1);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaError_t e = cudaStreamIsCapturing(s, &cs);
        if (e != cudaSuccess) return set_error((int)e, "spark_linear_noalloc: %s", cudaGetErrorString(e));
        SPARK_REQUIRE(cs == cudaStreamCaptureStatusNone, SPARK_ERR_INVALID,
                      "spark_linear_noalloc: the first call on device %d sets up its scratch and must come before "
                      "any stream capture",
                      dev);
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(e != cudaSuccess ? (int)e : SPARK_ERR_DEVICE, "spark_linear_noalloc: scratch lookup: %s",
                             cudaGetErrorString(e));
        e = cudaMemsetAsync(p, 0, ws_layout(0, 0).partials, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return set_error((int)e, "spark_linear_noalloc: scratch clear: %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return SPARK_OK;
}

}  // namespace
}  // namespace spark

extern "C" int spark_linear_noalloc(int fmt, const uint8_t* wq, const uint8_t* scales, const void* x, int x_dtype,
                                    int64_t M, int64_t oc, int64_t ic, int64_t ldx, const void* bias, int bias_dtype,
                                    void* y, int y_dtype, int64_t ldy, void* stream) {
    SPARK_REQUIRE(ic >= 0, SPARK_ERR_INVALID, "spark_linear_noalloc: negative size");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error((int)e, "spark_linear_noalloc: %s", cudaGetErrorString(e));
    // the larger of the two routes' needs (decode GEMV and tcgen05 GEMM), so
    // the check does not depend on which kernel spark_linear picks
    SPARK_REQUIRE(M >= 0 && oc >= 0, SPARK_ERR_INVALID, "spark_linear_noalloc: negative size");
    const size_t need = spark_linear_workspace_size(fmt & 0xff, M, oc, ic);
    SPARK_REQUIRE(need <= kNoAllocScratchBytes, SPARK_ERR_WORKSPACE,
                  "spark_linear_noalloc: M = %lld, ic = %lld needs %zu bytes of scratch, above the static %zu bytes "
                  "(use spark_linear with a caller-provided workspace)",
                  (long long)M, (long long)ic, need, kNoAllocScratchBytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    void* scratch = nullptr;
    const int rc = noalloc_scratch(dev, s, &scratch);
    if (rc) return rc;
    return spark_linear(fmt, wq, scales, x, x_dtype, M, oc, ic, ldx, bias, bias_dtype, y, y_dtype, ldy, scratch,
                        kNoAllocScratchBytes, stream);
}
