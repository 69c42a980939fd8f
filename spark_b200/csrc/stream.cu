// stream.cu -- persistent decode GEMV over a batch of packed linears
// (M <= 16 tokens, bf16 activations, fragment-major "tiled" weights).
//
// y_k[M, oc_k] = x_k[M, ic_k] . decode(W_k)^T (+ bias_k) for every op k of a
// batch, in ONE launch of one CTA per SM.  The work is HBM-bound at decode
// batch sizes, so the design keeps the weight stream running from the first
// op to the last:
//   * a producer thread copies every op's weight units, op after op, into a
//     5-stage shared-memory ring with bulk copies (evict-first in L2); an op
//     boundary is only a different source address for the next stage;
//   * 16 consumer warps each take one unit (16 rows x 256 columns) per stage,
//     decode it in registers and feed mma.sync; a row group split between
//     warps is summed deterministically (partials + counter, last arriver
//     adds in unit order);
//   * a preparation warp turns the activations of SPFP2 ops (up to 4 tokens)
//     into the fp8 operands described below; ops may depend on earlier ops'
//     outputs (device-side completion counters, bounded waits).
//
// SPFP2 on the fp8 tensor path (block_fp2_emu.py:36, :270-308).  A decoded
// SPFP2 weight is +-2^(e-10), e in [0, 15], or 0: exact in e5m2 (exponent
// field e + 5, no mantissa bits), so one byte permute of the block's table
// [e5m2(+), e5m2(-), 0, 0] turns four 2-bit codes into four A-operand bytes
// of mma.m16n8k32.e5m2.e4m3.  The activations are split per token into four
// e4m3 parts, x = sigma * (p0 + p1/16 + p2/256 + p3/4096) with sigma a power
// of two (max|x|/sigma in [128, 256)); each part is an N column of the MMA
// (the columns a 1-token GEMV would waste), every product is exact, and the
// epilogue adds the part columns with their powers of two.  Every bf16 value
// x with |x| >= 2^-10 max|x| is represented exactly; smaller ones to within
// 2^-24 max|x|, below the fp32 rounding of the accumulation.  Activations
// with a non-finite value (or a max outside 2^+-100) take the bf16 path.
//
// bf16 path (FP3, NVFP4, and SPFP2 above 4 tokens): the decoded weights are
// exact in bf16 (FP3 / e2m1 codes have <= 2 significant bits, e4m3 scales
// <= 4, SPFP2 values are powers of two) and mma.m16n8k16.bf16 reads the
// caller's x directly.
//
// Tiled layouts (spark_tile_weights): per unit, thread (g, t) of a warp owns
// the 64-column chunk [64t, 64t + 64) of rows g and g + 8, stored as
// lane-interleaved 16-byte vectors plus an 8-byte tail.  SPFP2: words 0-7
// hold, per 8-column block s of the chunk, the 8 codes of row g (low half)
// and row g + 8 (high half) with block column i at bits 4i and column 4 + i
// at bits 4i + 2; words 8-9 hold the 16 block exponents, byte s % 4 of word
// 8 + s / 4 = e(row g) | e(row g + 8) << 4.  FP3 / NVFP4: the reference
// layout's code words of the chunk and its scale word, per row.
#include <algorithm>
#include <mutex>
#include <new>

#include "common.cuh"

namespace spark {
namespace stream {

constexpr int kCW = 14;                       // consumer warps (16 warps in all: 128 registers a thread)
constexpr int kProdWarp = kCW;                // producer (lane 0 issues the copies)
constexpr int kPrepWarp = kCW + 1;            // activation preparation
constexpr int kThreads = (kCW + 2) * 32;
constexpr int kStages = 6;
constexpr int kSlotBytes = 2304;              // largest tiled unit (NVFP4)
constexpr int kStageBytes = kCW * kSlotBytes;
constexpr int kMaxOps = 48;
constexpr int kMaxSlots = 8;
constexpr int kMaxTok = 16;
constexpr int kF8Tok = 4;                     // tokens the fp8 path serves
constexpr int kParts = 4;                     // e4m3 parts per token
constexpr int kPartRing = 4;                  // partial-sum areas, reused every kPartRing ops
constexpr uint64_t kWaitNs = 2000000000ull;   // bounded waits: 2 s

// Control block inside the caller's workspace (bytes; the error word is at 0).
constexpr size_t kCtlAbort = 4;
constexpr size_t kCtlCtaDone = 8;
constexpr size_t kCtlOpDone = 64;                                   // int[kMaxOps]
constexpr size_t kCtlSlotCnt = kCtlOpDone + 4 * kMaxOps;            // int[kMaxSlots][2]
constexpr size_t kCtlSlotFlag = kCtlSlotCnt + 8 * kMaxSlots;        // int[kMaxSlots]
constexpr size_t kCtlSlotMax = kCtlSlotFlag + 4 * kMaxSlots;        // uint[kMaxSlots][kF8Tok]
constexpr size_t kCtlEnd = kCtlSlotMax + 4 * kMaxSlots * kF8Tok;
static_assert(kCtlEnd <= 4096, "control block overflows its 4 KB");

struct Op {
    const uint8_t* w;        // tiled weight
    const uint16_t* x;       // bf16 [M][ldx]
    void* y;
    const void* bias;
    int64_t ldx, ldy;
    int fmt, slot;           // slot >= 0: SPFP2 on the fp8 path (x prepared in that slot)
    int oc, n_kc, units, unit_bytes;
    int cnt_off, dep0, dep1, y_dtype;
    int bias_dtype, silu, n_rg, q;       // q, rem: units per virtual warp (see "work split")
    int rem, pad0, pad1, pad2;
};

struct Slot {
    const uint16_t* x;
    int64_t ldx;
    int64_t parts_off;       // bytes from Args::parts
    int ic, dep0, dep1, pad;
};

struct Args {
    Op op[kMaxOps];
    Slot slot[kMaxSlots];
    int n_ops, n_slots, M, ntf;   // ntf: n-tiles of the fp8 path (ceil(4 M / 8))
    int n_cnt, pad2;              // row-group counters used by the batch
    uint8_t* ws;
    int* counters;
    float* partials;
    int64_t part_stride;          // floats per ring area: T * 2 * M * 16
    uint8_t* parts;
};

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
__device__ __forceinline__ void mma_f8(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.f32.e5m2.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
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
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(20000u)
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
__device__ __forceinline__ int atom_acq_rel_add(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// Bounded wait on a shared-memory barrier phase, all lanes of the warp.
// False (and the abort flag raised) once kWaitNs pass, or when another warp
// has raised the abort flag.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* s_abort, volatile int* g_abort,
                                           int* err) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t dl = globaltimer_ns() + kWaitNs;
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*s_abort || *g_abort) return false;
        if (globaltimer_ns() > dl) {
            report_device_error(err, 1);
            *s_abort = 1;
            *g_abort = 1;
            return false;
        }
    }
}

// Bounded wait (one thread) until a device counter reaches `target`.
__device__ __forceinline__ bool wait_count(const int* p, int target, volatile int* abort, int* err) {
    if (ld_acquire(p) >= target) return true;
    const uint64_t dl = globaltimer_ns() + kWaitNs;
    while (true) {
        __nanosleep(100);
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
// Op k's units are split evenly over T = G * kCW virtual warps in unit
// order: virtual warp v holds q + (v < rem) units starting at
// v * q + min(v, rem) (q = U / T, rem = U % T, computed on the host).  CTA c
// runs virtual warps v = w' * G + c' (c' = (c + k) % G, w' = (w + k) % kCW for
// its consumer warp w), so every CTA gets an equal share (at most one unit
// apart) and the roles rotate from op to op.  Row-group contributors are then a
// contiguous range of virtual warps: sub-ranges are empty only when q == 0,
// and then only for v >= rem, after every non-empty one.
__device__ __forceinline__ int vw_start(const Op& op, int v) { return v * op.q + min(v, op.rem); }
__device__ __forceinline__ int vw_size(const Op& op, int v) { return op.q + (v < op.rem ? 1 : 0); }
__device__ __forceinline__ int vw_owner(const Op& op, int u) {
    const int big = op.rem * (op.q + 1);
    return u < big ? u / (op.q + 1) : op.rem + (u - big) / op.q;
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
// e4m3 scale (exact in bf16).
template <int FMT>
__device__ __forceinline__ void decode_scaled(const uint32_t* c, uint32_t scale_word, int s, const uint32_t* pair_tab,
                                              const uint32_t* scale_tab, uint32_t* A) {
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

// SPFP2 stream layout, bf16 pairs of one row for block s: codes c0..c3 are the
// nibbles of sA (low 16 bits), c4..c7 those of sB; e the block exponent.
// bf16 of +-2^(e-10): biased exponent E = 117 + e, high byte sign | E >> 1,
// low byte (E & 1) << 7.  Out: P[0..3] = column pairs (0,1) (2,3) (4,5) (6,7).
__device__ __forceinline__ void decode_spfp2_bf16(uint32_t sA, uint32_t sB, uint32_t e, uint32_t* P) {
    const uint32_t E = 117u + e;
    const uint32_t TH = (E >> 1) * 0x101u + 0x8000u;     // [H, H | 0x80, 0, 0]
    const uint32_t TL = (E & 1u) * 0x8080u;              // [L, L, 0, 0]
    const uint32_t hA = prmt(TH, 0u, sA), lA = prmt(TL, 0u, sA);
    const uint32_t hB = prmt(TH, 0u, sB), lB = prmt(TL, 0u, sB);
    P[0] = prmt(lA, hA, 0x5140u);
    P[1] = prmt(lA, hA, 0x7362u);
    P[2] = prmt(lB, hB, 0x5140u);
    P[3] = prmt(lB, hB, 0x7362u);
}

template <int FMT>
__host__ __device__ constexpr int frag_words() {
    return FMT == SPARK_FMT_SPFP2 ? 10 : (FMT == SPARK_FMT_FP3 ? 14 : 18);
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

// ---------------------------------------------------------------- epilogue
// A lane's values of one row group: v[idx][r] for rows g (r = 0) and g + 8
// (r = 1).  fp8 path (F8): idx = n-tile j, token 2j + (t >> 1), held by the
// lanes with even t; bf16 path: idx = 2j + i, token 8j + 2t + i.
template <bool F8>
__device__ __forceinline__ int val_token(int idx, int t) {
    return F8 ? 2 * idx + (t >> 1) : 8 * (idx >> 1) + 2 * t + (idx & 1);
}

__device__ __forceinline__ float bias_at(const Op& op, int64_t row) {
    return op.bias ? load_as_float(op.bias, op.bias_dtype, row) : 0.0f;
}

// per-token output scale: the fp8 path's power of two, 1 on the bf16 path
__device__ __forceinline__ float tok_scale(const float4& sc, int m) {
    return m == 0 ? sc.x : (m == 1 ? sc.y : (m == 2 ? sc.z : sc.w));
}

template <bool F8, int NV>
__device__ __forceinline__ void write_rows(const Op& op, int M, int rg, const float (&v)[NV][2], const float4& sc,
                                           int g, int t) {
    if (F8 && (t & 1)) return;
    const int64_t r0 = (int64_t)rg * 16 + g, r1 = r0 + 8;
    if (op.silu) {
        const float bg = bias_at(op, r0), bu = bias_at(op, r1);
#pragma unroll
        for (int idx = 0; idx < NV; ++idx) {
            const int m = val_token<F8>(idx, t);
            if (m >= M) continue;
            const float s = F8 ? tok_scale(sc, m) : 1.0f;
            const float gv = v[idx][0] * s + bg, uv = v[idx][1] * s + bu;
            store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + (int64_t)rg * 8 + g,
                             gv / (1.0f + __expf(-gv)) * uv);
        }
        return;
    }
    const float b0 = r0 < op.oc ? bias_at(op, r0) : 0.0f, b1 = r1 < op.oc ? bias_at(op, r1) : 0.0f;
#pragma unroll
    for (int idx = 0; idx < NV; ++idx) {
        const int m = val_token<F8>(idx, t);
        if (m >= M) continue;
        const float s = F8 ? tok_scale(sc, m) : 1.0f;
        if (r0 < op.oc) store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r0, v[idx][0] * s + b0);
        if (r1 < op.oc) store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r1, v[idx][1] * s + b1);
    }
}

// ---------------------------------------------------------------- consumer state
struct Ctl {
    int* err;
    volatile int* abort;
    int* op_done;
    int* slot_cnt;
    int* slot_flag;
    unsigned* slot_max;
};

__device__ __forceinline__ Ctl ctl_of(uint8_t* ws) {
    Ctl c;
    c.err = reinterpret_cast<int*>(ws);
    c.abort = reinterpret_cast<volatile int*>(ws + kCtlAbort);
    c.op_done = reinterpret_cast<int*>(ws + kCtlOpDone);
    c.slot_cnt = reinterpret_cast<int*>(ws + kCtlSlotCnt);
    c.slot_flag = reinterpret_cast<int*>(ws + kCtlSlotFlag);
    c.slot_max = reinterpret_cast<unsigned*>(ws + kCtlSlotMax);
    return c;
}

// power-of-two scale sigma of a token: max|x| / sigma in [128, 256)
__device__ __forceinline__ int token_exp(unsigned maxbits) {
    return (int)((maxbits >> 23) & 0xffu) - 127 - 7;
}

// Flush the row-group segment [seg0, seg1) of op k held in v: write the rows
// when the segment is the whole row group, else publish the partial; the
// last contributor sums the partials in unit order and writes the rows.
template <bool F8, int NV>
__device__ __noinline__ void flush(const Args& a, const Ctl& C, int k, int vw, int rg, int seg0, int seg1, int u_first,
                                   const float (&v)[NV][2], float4 sc, int lane) {
    const Op& op = a.op[k];
    const int g = lane >> 2, t = lane & 3;
    const int K = op.n_kc, M = a.M;
    if (seg0 == rg * K && seg1 == (rg + 1) * K) {
        write_rows<F8, NV>(op, M, rg, v, sc, g, t);
        return;
    }
    const int T = gridDim.x * kCW;
    float* area = a.partials + (int64_t)(k % kPartRing) * a.part_stride;
    // areas are reused every kPartRing ops: the op that last used this one
    // must be finished (every warp past it, its partials read)
    if (k >= kPartRing) {
        bool ok = true;
        if (lane == 0) ok = wait_count(C.op_done + (k - kPartRing), T, C.abort, C.err);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
    }
    const int slot = (seg0 / K == u_first / K) ? 0 : 1;
    float* mine = area + ((int64_t)vw * 2 + slot) * M * 16;
    if (!(F8 && (t & 1))) {
#pragma unroll
        for (int idx = 0; idx < NV; ++idx) {
            const int m = val_token<F8>(idx, t);
            if (m < M) {
                __stcg(mine + m * 16 + g, v[idx][0]);
                __stcg(mine + m * 16 + g + 8, v[idx][1]);
            }
        }
    }
    __threadfence();
    __syncwarp();
    const int first = rg * K;
    const int v_lo = vw_owner(op, first), v_hi = vw_owner(op, first + K - 1);
    int old = 0;
    if (lane == 0) old = atom_acq_rel_add(a.counters + op.cnt_off + rg, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != v_hi - v_lo) return;
    __threadfence();
    // the first contributor holds this row group in its second slot when its
    // sub-range began in an earlier row group
    const bool lo_second = vw_start(op, v_lo) < first;
    // lane l sums row (l & 15) of tokens (l >> 4) + 2i
    const int row = lane & 15;
    float sum[kMaxTok / 2];
#pragma unroll
    for (int i = 0; i < kMaxTok / 2; ++i) sum[i] = 0.0f;
    for (int w = v_lo; w <= v_hi; ++w) {
        const float* src = area + ((int64_t)w * 2 + ((w == v_lo && lo_second) ? 1 : 0)) * M * 16;
#pragma unroll
        for (int i = 0; i < kMaxTok / 2; ++i) {
            const int m = (lane >> 4) + 2 * i;
            if (m < M) sum[i] += __ldcg(src + m * 16 + row);
        }
    }
    if (lane == 0) a.counters[op.cnt_off + rg] = 0;
    const int64_t r = (int64_t)rg * 16 + row;
    if (op.silu) {
        // rows 0-7 of the group are gate rows, 8-15 the matching up rows
        float up[kMaxTok / 2];
#pragma unroll
        for (int i = 0; i < kMaxTok / 2; ++i) up[i] = __shfl_down_sync(0xffffffffu, sum[i], 8);
        if (row < 8) {
            const float bg = bias_at(op, r), bu = bias_at(op, r + 8);
#pragma unroll
            for (int i = 0; i < kMaxTok / 2; ++i) {
                const int m = (lane >> 4) + 2 * i;
                if (m >= M) continue;
                const float s = F8 ? tok_scale(sc, m) : 1.0f;
                const float gv = sum[i] * s + bg, uv = up[i] * s + bu;
                store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + (int64_t)rg * 8 + row,
                                 gv / (1.0f + __expf(-gv)) * uv);
            }
        }
        return;
    }
    if (r < op.oc) {
        const float b = bias_at(op, r);
#pragma unroll
        for (int i = 0; i < kMaxTok / 2; ++i) {
            const int m = (lane >> 4) + 2 * i;
            if (m < M) store_from_float(op.y, op.y_dtype, (int64_t)m * op.ldy + r, sum[i] * (F8 ? tok_scale(sc, m) : 1.0f) + b);
        }
    }
}

// ---------------------------------------------------------------- unit kernels
// fp8 path: one SPFP2 unit (8 blocks per row, rows g and g + 8) into acc.
template <int NTF>
__device__ __forceinline__ void unit_spfp2_f8(const uint32_t* fw, const uint2 (&b)[8][NTF],
                                              float (&acc)[2][NTF][4]) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const uint32_t E = fw[8 + (s >> 2)];
        // e5m2 of +2^(e-10) is (e + 5) << 2: four blocks' bytes per word, and
        // their negatives; one permute picks the block's [+, -, 0, 0] table
        const uint32_t PL = (E & 0x0f0f0f0fu) * 4u + 0x14141414u;
        const uint32_t PH = ((E >> 4) & 0x0f0f0f0fu) * 4u + 0x14141414u;
        const uint32_t sel = 0x8800u | ((4u + (uint32_t)(s & 3)) << 4) | (uint32_t)(s & 3);
        const uint32_t Tg = prmt(PL, PL | 0x80808080u, sel);
        const uint32_t Th = prmt(PH, PH | 0x80808080u, sel);
        const uint32_t W = fw[s];
        const uint32_t x0 = W & 0x33333333u, x1 = (W >> 2) & 0x33333333u;
        const uint32_t a0 = prmt(Tg, 0u, x0), a2 = prmt(Tg, 0u, x1);
        const uint32_t a1 = prmt(Th, 0u, x0 >> 16), a3 = prmt(Th, 0u, x1 >> 16);
#pragma unroll
        for (int j = 0; j < NTF; ++j) mma_f8(acc[s & 1][j], a0, a1, a2, a3, b[s][j].x, b[s][j].y);
    }
}

// bf16 path: one unit of any format; x rows read directly (16 bytes per step).
template <int FMT, int NTB>
__device__ __forceinline__ void unit_bf16(const uint32_t* fw, const uint16_t* const (&xr)[NTB], const bool (&xv)[NTB],
                                          int64_t col, const uint32_t* pair_tab, const uint32_t* scale_tab,
                                          float (&acc)[2][NTB][4]) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t A0[4], A1[4];
        if constexpr (FMT == SPARK_FMT_SPFP2) {
            const uint32_t W = fw[s];
            const uint32_t E = fw[8 + (s >> 2)] >> (8 * (s & 3));
            const uint32_t sA = W & 0x3333u, sB = (W >> 2) & 0x3333u;
            decode_spfp2_bf16(sA, sB, E & 0xfu, A0);
            decode_spfp2_bf16((W >> 16) & 0x3333u, (W >> 18) & 0x3333u, (E >> 4) & 0xfu, A1);
        } else {
            constexpr int CW = FMT == SPARK_FMT_FP3 ? 6 : 8;
            decode_scaled<FMT>(fw, fw[CW], s, pair_tab, scale_tab, A0);
            decode_scaled<FMT>(fw + CW + 1, fw[2 * CW + 1], s, pair_tab, scale_tab, A1);
        }
#pragma unroll
        for (int j = 0; j < NTB; ++j) {
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (xv[j]) x = ldg_nc_v4(xr[j] + col + 8 * s);
            mma_bf16(acc[0][j], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
            mma_bf16(acc[1][j], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
        }
    }
}

// ---------------------------------------------------------------- roles
__device__ void producer(const Args& a, uint8_t* ring, uint64_t* full, uint64_t* empty, const Ctl& C,
                         volatile int* s_abort) {
    const int G = gridDim.x, c = blockIdx.x;
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    uint32_t q = 0;
    bool stop = false;
    for (int k = 0; k < a.n_ops && !stop; ++k) {
        const Op& op = a.op[k];
        const int cr = (c + k) % G;
        const int S = op.q + (cr < op.rem ? 1 : 0);
        for (int s = 0; s < S; ++s, ++q) {
            const uint32_t st = q % kStages;
            if (!wait_phase(smem_u32(empty + st), ((q / kStages) & 1u) ^ 1u, s_abort, C.abort, C.err) || *C.abort) {
                *s_abort = 1;
                stop = true;
                break;
            }
            // warps whose sub-range is one unit longer hold the last stage's units
            int n_here = kCW;
            if (s == op.q) {
                n_here = 0;
#pragma unroll 1
                for (int w = 0; w < kCW; ++w) n_here += ((w + k) % kCW) * G + cr < op.rem ? 1 : 0;
            }
            const uint32_t fb = smem_u32(full + st);
            mbar_expect_tx(fb, (uint32_t)(n_here * op.unit_bytes));
#pragma unroll 1
            for (int w = 0; w < kCW; ++w) {
                const int v = ((w + k) % kCW) * G + cr;
                if (s >= vw_size(op, v)) continue;
                const uint8_t* src = op.w + (int64_t)(vw_start(op, v) + s) * op.unit_bytes;
                const uint32_t dst = smem_u32(ring + st * kStageBytes + w * kSlotBytes);
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
                    "%2, [%3], %4;" ::"r"(dst),
                    "l"(src), "r"((uint32_t)op.unit_bytes), "r"(fb), "l"(policy)
                    : "memory");
            }
        }
    }
    if (stop) {
        // let the copies already issued land before the CTA retires
        const uint32_t lo = q > kStages ? q - kStages : 0;
        for (uint32_t p = lo; p < q; ++p) {
            const uint32_t st = p % kStages;
            const uint64_t dl = globaltimer_ns() + kWaitNs;
            while (!mbar_try(smem_u32(full + st), (p / kStages) & 1u) && globaltimer_ns() < dl) {
            }
        }
    }
}

// Activation preparation for the fp8 path: per slot, every CTA takes a slice
// of 8-column blocks; pass 1 publishes the per-token max |x|, pass 2 (after
// all CTAs) writes the e4m3 parts in the order the consumers' B fragments
// read them.
__device__ void prepare(const Args& a, const Ctl& C, int lane) {
    const int G = gridDim.x, c = blockIdx.x;
    const int M = a.M;
    for (int sl = 0; sl < a.n_slots; ++sl) {
        const Slot& S = a.slot[sl];
        bool ok = true;
        if (lane == 0) {
            if (S.dep0 >= 0) ok = wait_count(C.op_done + S.dep0, G * kCW, C.abort, C.err);
            if (ok && S.dep1 >= 0) ok = wait_count(C.op_done + S.dep1, G * kCW, C.abort, C.err);
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
        const int nb = S.ic / 8;
        const int b0 = (int)((int64_t)nb * c / G), b1 = (int)((int64_t)nb * (c + 1) / G);
        float mx[kF8Tok];
        int bad = 0;
#pragma unroll
        for (int m = 0; m < kF8Tok; ++m) {
            mx[m] = 0.0f;
            if (m >= M) continue;
            for (int b = b0 + lane; b < b1; b += 32) {
                const uint4 q = *reinterpret_cast<const uint4*>(S.x + (int64_t)m * S.ldx + 8 * b);
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = fabsf(__uint_as_float(w4[i] << 16)), hi = fabsf(__uint_as_float(w4[i] & 0xffff0000u));
                    bad |= !(lo <= 3.4028235e38f) | !(hi <= 3.4028235e38f);
                    mx[m] = fmaxf(mx[m], fmaxf(lo, hi));
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], o));
        }
        bad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
            for (int m = 0; m < M && m < kF8Tok; ++m) atomicMax(C.slot_max + sl * kF8Tok + m, __float_as_uint(mx[m]));
            if (bad) atomicOr(C.slot_flag + sl, 1);
            __threadfence();
            red_release_add(C.slot_cnt + 2 * sl, 1);
            ok = wait_count(C.slot_cnt + 2 * sl, G, C.abort, C.err);
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return;
        __threadfence();
        int flag = __ldcg(C.slot_flag + sl);
        float up[kF8Tok];
#pragma unroll
        for (int m = 0; m < kF8Tok; ++m) {
            up[m] = 1.0f;
            if (m >= M) continue;
            const unsigned mb = __ldcg(C.slot_max + sl * kF8Tok + m);
            if (mb == 0u) continue;                       // all zero: parts are zero for any scale
            const int ex = token_exp(mb);
            if (ex < -100 || ex > 100) flag = 1;          // (subnormal maxima included)
            else up[m] = __uint_as_float((uint32_t)(127 - ex) << 23);
        }
        if (!flag) {
            const int ntf = a.ntf;
            uint8_t* parts = a.parts + S.parts_off;
#pragma unroll 1
            for (int m = 0; m < M && m < kF8Tok; ++m)
                for (int b = b0 + lane; b < b1; b += 32) {
                    const uint4 q = *reinterpret_cast<const uint4*>(S.x + (int64_t)m * S.ldx + 8 * b);
                    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
                    float r[8];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        r[2 * i] = __uint_as_float(w4[i] << 16) * up[m];
                        r[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u) * up[m];
                    }
                    // column 8b: unit kc, thread t of the chunk, block s within it
                    const int col = 8 * b, kc = col >> 8, o = col & 255, t = o >> 6, s = (o & 63) >> 3;
                    uint8_t* base = parts + (int64_t)kc * 2048 * ntf + (int64_t)s * 8 * ntf * 32 + t * 8;
#pragma unroll
                    for (int p = 0; p < kParts; ++p) {
                        uint32_t lo = 0u, hi = 0u;
                        const float sc = __uint_as_float((uint32_t)(127 + 4 * p) << 23);   // 2^(4p)
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t e = f32_to_e4m3(r[i] * sc);
                            r[i] -= e4m3_to_f32(e) / sc;           // exact: e has <= 4 bits of r's
                            if (i < 4) lo |= e << (8 * i);
                            else hi |= e << (8 * (i - 4));
                        }
                        const int n = kParts * m + p;
                        *reinterpret_cast<uint2*>(base + (int64_t)n * 32) = make_uint2(lo, hi);
                    }
                }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_add(C.slot_cnt + 2 * sl + 1, 1);
    }
}

template <int NTF, int NTB>
__device__ void consumer(const Args& a, const uint8_t* ring, uint64_t* full, uint64_t* empty, const Ctl& C,
                         volatile int* s_abort, const uint32_t* pair_fp3, const uint32_t* pair_nv,
                         const uint32_t* scale_tab, int warp, int lane) {
    const int G = gridDim.x, c = blockIdx.x;
    const int T = G * kCW;
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M;
    uint32_t q = 0;
    bool dead = false;
    for (int k = 0; k < a.n_ops; ++k) {
        const Op& op = a.op[k];
        const int cr = (c + k) % G;
        const int vw = ((warp + k) % kCW) * G + cr;
        const int u0 = vw_start(op, vw), mine = vw_size(op, vw);
        const int S = op.q + (cr < op.rem ? 1 : 0);
        // inputs: earlier ops this op reads, and the prepared fp8 activations
        bool f8 = false;
        float4 sc = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if (mine > 0 && !dead) {
            bool ok = true;
            if (lane == 0) {
                if (op.dep0 >= 0) ok = wait_count(C.op_done + op.dep0, T, C.abort, C.err);
                if (ok && op.dep1 >= 0) ok = wait_count(C.op_done + op.dep1, T, C.abort, C.err);
                if (ok && op.slot >= 0) ok = wait_count(C.slot_cnt + 2 * op.slot + 1, G, C.abort, C.err);
            }
            dead = !__shfl_sync(0xffffffffu, ok ? 1 : 0, 0);
            if (!dead && op.slot >= 0 && __ldcg(C.slot_flag + op.slot) == 0) {
                f8 = true;
                float s4[kF8Tok];
#pragma unroll
                for (int m = 0; m < kF8Tok; ++m) {
                    const unsigned mb = m < M ? __ldcg(C.slot_max + op.slot * kF8Tok + m) : 0u;
                    s4[m] = mb ? __uint_as_float((uint32_t)(127 + token_exp(mb)) << 23) : 1.0f;
                }
                sc = make_float4(s4[0], s4[1], s4[2], s4[3]);
            }
        }
        int kc = mine > 0 ? u0 % op.n_kc : 0, rg = mine > 0 ? u0 / op.n_kc : 0;
        int seg0 = u0;
        float accf[2][NTF][4];
        float accb[2][NTB][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int j = 0; j < NTF; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) accf[h][j][i] = 0.0f;
#pragma unroll
            for (int j = 0; j < NTB; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) accb[h][j][i] = 0.0f;
        }
        const uint8_t* parts_base = f8 ? a.parts + a.slot[op.slot].parts_off : nullptr;
        for (int s = 0; s < S; ++s, ++q) {
            const uint32_t st = q % kStages;
            const bool have = s < mine;
            // B operands of the fp8 path first: their loads overlap the stage wait
            uint2 bq[8][NTF];
            if (f8 && have) {
                const uint8_t* pb = parts_base + (int64_t)kc * 2048 * NTF + ((g * 4 + t) << 3);
#pragma unroll
                for (int ss = 0; ss < 8; ++ss)
#pragma unroll
                    for (int j = 0; j < NTF; ++j)
                        bq[ss][j] = (8 * j + g < kParts * M) ? ldg_v2(pb + (ss * 8 * NTF + 8 * j) * 32)
                                                             : make_uint2(0u, 0u);
            }
            if (!dead) {
                const bool ok = __all_sync(0xffffffffu, wait_phase(smem_u32(full + st), (q / kStages) & 1u, s_abort,
                                                                   C.abort, C.err));
                if (!ok) dead = true;
            }
            uint32_t fw[18];
            if (have && !dead) {
                const uint8_t* slot = ring + st * kStageBytes + warp * kSlotBytes;
                if (op.fmt == SPARK_FMT_SPFP2) load_frag<10>(slot, lane, fw);
                else if (op.fmt == SPARK_FMT_FP3) load_frag<14>(slot, lane, fw);
                else load_frag<18>(slot, lane, fw);
            }
            __syncwarp();
            if (lane == 0 && !dead) mbar_arrive(smem_u32(empty + st));
            if (!have || dead) continue;

            if (f8) {
                unit_spfp2_f8<NTF>(fw, bq, accf);
            } else {
                const uint16_t* xr[NTB];
                bool xv[NTB];
#pragma unroll
                for (int j = 0; j < NTB; ++j) {
                    xv[j] = 8 * j + g < M;
                    xr[j] = op.x + (int64_t)(8 * j + g) * op.ldx;
                }
                const int64_t col = (int64_t)kc * 256 + t * 64;
                if (op.fmt == SPARK_FMT_SPFP2) unit_bf16<SPARK_FMT_SPFP2, NTB>(fw, xr, xv, col, pair_fp3, scale_tab, accb);
                else if (op.fmt == SPARK_FMT_FP3) unit_bf16<SPARK_FMT_FP3, NTB>(fw, xr, xv, col, pair_fp3, scale_tab, accb);
                else unit_bf16<SPARK_FMT_NVFP4, NTB>(fw, xr, xv, col, pair_nv, scale_tab, accb);
            }
            const int u = u0 + s;
            if (kc == op.n_kc - 1 || s + 1 == mine) {
                if (f8) {
                    // columns 8j + 2t, 8j + 2t + 1 hold parts 2(t & 1), 2(t & 1) + 1
                    // of token 2j + (t >> 1): scale by 2^-4p, add the lane pair
                    const float s0 = (t & 1) ? 1.0f / 256.0f : 1.0f, s1 = (t & 1) ? 1.0f / 4096.0f : 1.0f / 16.0f;
                    float vals[NTF][2];
#pragma unroll
                    for (int j = 0; j < NTF; ++j) {
                        float vg = (accf[0][j][0] + accf[1][j][0]) * s0 + (accf[0][j][1] + accf[1][j][1]) * s1;
                        float vh = (accf[0][j][2] + accf[1][j][2]) * s0 + (accf[0][j][3] + accf[1][j][3]) * s1;
                        vals[j][0] = vg + __shfl_xor_sync(0xffffffffu, vg, 1);
                        vals[j][1] = vh + __shfl_xor_sync(0xffffffffu, vh, 1);
                    }
                    flush<true, NTF>(a, C, k, vw, rg, seg0, u + 1, u0, vals, sc, lane);
                } else {
                    float vals[2 * NTB][2];
#pragma unroll
                    for (int j = 0; j < NTB; ++j)
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            vals[2 * j + i][0] = accb[0][j][i] + accb[1][j][i];
                            vals[2 * j + i][1] = accb[0][j][2 + i] + accb[1][j][2 + i];
                        }
                    flush<false, 2 * NTB>(a, C, k, vw, rg, seg0, u + 1, u0, vals, sc, lane);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
#pragma unroll
                    for (int j = 0; j < NTF; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) accf[h][j][i] = 0.0f;
#pragma unroll
                    for (int j = 0; j < NTB; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) accb[h][j][i] = 0.0f;
                }
                seg0 = u + 1;
            }
            if (++kc == op.n_kc) {
                kc = 0;
                ++rg;
            }
        }
        // this warp is done with op k (outputs and partial reads included)
        __syncwarp();
        if (lane == 0) {
            __threadfence();
            red_release_add(C.op_done + k, 1);
        }
    }
}

template <int NTF, int NTB>
__global__ void __launch_bounds__(kThreads, 1) k_stream(const __grid_constant__ Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint32_t* pair_fp3 = reinterpret_cast<uint32_t*>(empty + kStages);
    uint32_t* pair_nv = pair_fp3 + 64;
    uint32_t* scale_tab = pair_nv + 256;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Ctl C = ctl_of(a.ws);
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < kStages; ++i) {
            mbar_init(smem_u32(full + i), 1);
            mbar_init(smem_u32(empty + i), kCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const uint32_t sb = __float_as_uint(e4m3_to_f32((uint32_t)i)) >> 16;   // e4m3 values are exact in bf16
        scale_tab[i] = sb | (sb << 16);
        pair_nv[i] = code_bf16(SPARK_FMT_NVFP4, (uint32_t)i & 15u) | (code_bf16(SPARK_FMT_NVFP4, (uint32_t)i >> 4) << 16);
        if (i < 64) pair_fp3[i] = code_bf16(SPARK_FMT_FP3, (uint32_t)i & 7u) | (code_bf16(SPARK_FMT_FP3, (uint32_t)i >> 3) << 16);
    }
    __syncthreads();
    volatile int* sab = &s_abort;
    if (warp == kProdWarp) {
        if (lane == 0) producer(a, ring, full, empty, C, sab);
    } else if (warp == kPrepWarp) {
        prepare(a, C, lane);
    } else {
        consumer<NTF, NTB>(a, ring, full, empty, C, sab, pair_fp3, pair_nv, scale_tab, warp, lane);
    }
    __syncthreads();
    // the last CTA out returns the control block to zero for the next launch
    if (threadIdx.x == 0) {
        __threadfence();
        const int old = atomicAdd(reinterpret_cast<int*>(a.ws + kCtlCtaDone), 1);
        if (old == (int)gridDim.x - 1) {
            __threadfence();
            for (int k = 0; k < a.n_ops; ++k) C.op_done[k] = 0;
            for (int i = 0; i < 2 * kMaxSlots; ++i) C.slot_cnt[i] = 0;
            for (int i = 0; i < kMaxSlots; ++i) C.slot_flag[i] = 0;
            for (int i = 0; i < kMaxSlots * kF8Tok; ++i) C.slot_max[i] = 0u;
            // an aborted launch can leave row-group counters raised
            if (*C.abort)
                for (int i = 0; i < a.n_cnt; ++i) a.counters[i] = 0;
            *C.abort = 0;
            __threadfence();
            *reinterpret_cast<volatile int*>(a.ws + kCtlCtaDone) = 0;
        }
    }
}

constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 2 * kStages * 8 + (64 + 256 + 256) * 4;

int sm_count(int dev) {
    static int cache[64] = {};
    if (dev < 0 || dev >= 64) return 0;
    if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
    return cache[dev];
}

std::mutex g_mu;

template <int NTF, int NTB>
int launch(const Args& a, int grid, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    {
        static bool done[64] = {};
        std::lock_guard<std::mutex> lk(g_mu);
        if (!done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(k_stream<NTF, NTB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_stream<NTF, NTB>, a);
    if (e != cudaSuccess) return set_error((int)e, "k_stream launch: %s", cudaGetErrorString(e));
    return SPARK_OK;
}

}  // namespace stream

// ---------------------------------------------------------------- host entry (used by gemv.cu)
// Workspace layout shared with spark_linear: control block in [0, 4096), the
// row-group counters at `counters_off` (int[max_counters], self-resetting),
// then this kernel's partial sums and prepared activations from `scratch_off`.
struct StreamPlan {
    stream::Args args;
    size_t scratch_bytes = 0;   // bytes needed from scratch_off
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
    Args& a = P->args;
    a = Args{};
    a.n_ops = n_ops;
    a.M = (int)M;
    a.ntf = M <= 2 ? 1 : 2;
    const bool f8 = M <= kF8Tok;
    int64_t cnt = 0;
    int64_t parts_bytes = 0;
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
        p.n_rg = (int)((o.oc + 15) / 16);
        const int64_t units = (int64_t)p.n_rg * p.n_kc;
        SPARK_REQUIRE(units < (1ll << 30) && o.oc < (1ll << 30), SPARK_ERR_UNSUPPORTED,
                      "spark_linear_batch: op %d too large", k);
        p.units = (int)units;
        p.q = (int)(units / ((int64_t)G * kCW));
        p.rem = (int)(units % ((int64_t)G * kCW));
        p.unit_bytes = unit_bytes_of(fmt);
        p.cnt_off = (int)cnt;
        cnt += p.n_rg;
        p.dep0 = o.dep[0];
        p.dep1 = o.dep[1];
        p.y_dtype = o.y_dtype;
        p.bias_dtype = o.bias ? o.bias_dtype : 0;
        p.silu = silu ? 1 : 0;
        p.slot = -1;
        if (fmt == SPARK_FMT_SPFP2 && f8) {
            int sl = -1;
            for (int j = 0; j < a.n_slots; ++j) {
                const Slot& S = a.slot[j];
                if (S.x == p.x && S.ldx == p.ldx && S.ic == (int)o.ic && S.dep0 == p.dep0 && S.dep1 == p.dep1) sl = j;
            }
            if (sl < 0 && a.n_slots < kMaxSlots) {
                sl = a.n_slots++;
                Slot& S = a.slot[sl];
                S.x = p.x;
                S.ldx = p.ldx;
                S.ic = (int)o.ic;
                S.dep0 = p.dep0;
                S.dep1 = p.dep1;
                S.parts_off = parts_bytes;
                parts_bytes += (o.ic / 256) * 2048 * a.ntf;
            }
            p.slot = sl;     // -1 when the slots are used up: that op takes the bf16 path
        }
    }
    a.n_cnt = (int)std::min<int64_t>(cnt, max_counters);
    SPARK_REQUIRE(cnt <= max_counters, SPARK_ERR_UNSUPPORTED,
                  "spark_linear_batch: %lld row groups in the batch, above %lld", (long long)cnt, (long long)max_counters);
    const int64_t T = (int64_t)G * kCW;
    const int ring = n_ops < kPartRing ? n_ops : kPartRing;
    a.part_stride = T * 2 * M * 16;
    const size_t part_bytes = (size_t)ring * a.part_stride * sizeof(float);
    P->scratch_bytes = (part_bytes + 255) / 256 * 256 + (size_t)parts_bytes;
    P->grid = G;
    a.ws = ws;
    if (ws) {
        a.counters = reinterpret_cast<int*>(ws + counters_off);
        a.partials = reinterpret_cast<float*>(ws + scratch_off);
        a.parts = ws + scratch_off + (part_bytes + 255) / 256 * 256;
    }
    return SPARK_OK;
}

int stream_plan_alloc(StreamPlan** P) {
    *P = new (std::nothrow) StreamPlan();
    return *P ? SPARK_OK : set_error(SPARK_ERR_INVALID, "spark_linear_batch: out of host memory");
}
void stream_plan_free(StreamPlan* P) { delete P; }
size_t stream_plan_scratch(const StreamPlan* P) { return P->scratch_bytes; }

// scratch of a one-op batch (spark_linear on tiled weights, bf16 x)
size_t stream_scratch_single(int64_t M, int64_t ic) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t Mc = M < 1 ? 1 : (M > stream::kMaxTok ? stream::kMaxTok : M);
    const size_t part = (size_t)stream::sm_count(dev) * stream::kCW * 2 * Mc * 16 * sizeof(float);
    const size_t parts = Mc <= stream::kF8Tok ? (size_t)(ic / 256) * 2048 * (Mc <= 2 ? 1 : 2) : 0;
    return (part + 255) / 256 * 256 + parts;
}

int stream_launch(const StreamPlan& P, cudaStream_t s) {
    const stream::Args& a = P.args;
    if (a.M <= 2) return stream::launch<1, 1>(a, P.grid, s);
    if (a.M <= 4) return stream::launch<2, 1>(a, P.grid, s);
    if (a.M <= 8) return stream::launch<1, 1>(a, P.grid, s);
    return stream::launch<1, 2>(a, P.grid, s);
}

}  // namespace spark
