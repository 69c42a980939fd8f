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
//   * 15 consumer warps each take one unit (16 rows x 256 columns) per stage,
//     decode it in registers and feed mma.sync (bf16, fp32 accumulation); a
//     row group split between warps is summed deterministically (partials +
//     counter, the last arriver adds them in unit order);
//   * ops may read earlier ops' outputs: a consumer waits on device-side
//     completion counters (bounded waits) before it reads such an input, while
//     the op's weights are already streaming.
//
// Every decoded weight is exact in bf16 (SPFP2 values are powers of two,
// block_fp2_emu.py:36; FP3 / e2m1 codes have <= 2 significant bits and e4m3
// scales <= 4, fp3_emu.py:47, nvfp4_emu.py:109-123), so mma.m16n8k16.bf16
// reads the caller's bf16 x directly.
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

constexpr int kCW = 15;                       // consumer warps
constexpr int kProdWarp = kCW;                // producer (lane 0 issues the copies)
constexpr int kThreads = (kCW + 1) * 32;      // 16 warps: 128 registers a thread
constexpr int kStages = 5;
constexpr int kSlotBytes = 2304;              // largest tiled unit (NVFP4)
constexpr int kStageBytes = kCW * kSlotBytes;
constexpr int kMaxOps = 48;
constexpr int kMaxTok = 16;
constexpr size_t kPartAreaBudget = (size_t)16 << 20;   // partial-sum areas of a batch: one per op up to this
constexpr uint64_t kWaitNs = 2000000000ull;   // bounded waits: 2 s

// Control block inside the caller's workspace (bytes; the error word is at 0).
constexpr size_t kCtlAbort = 4;
constexpr size_t kCtlCtaDone = 8;
constexpr size_t kCtlOpDone = 64;             // int[kMaxOps]
static_assert(kCtlOpDone + 4 * kMaxOps <= 4096, "control block overflows its 4 KB");

struct Op {
    const uint8_t* w;        // tiled weight
    const uint16_t* x;       // bf16 [M][ldx]
    void* y;
    const void* bias;
    int64_t ldx, ldy;
    int fmt, oc, n_kc, units;
    int unit_bytes, cnt_off, dep0, dep1;
    int y_dtype, bias_dtype, silu, n_rg;
    int q, rem, waited, pad1;  // q, rem: units per virtual warp (see "work split"); waited: an op or a
                               // partial-area reuse waits for this op's completion count
};

struct Args {
    Op op[kMaxOps];
    int n_ops, M, n_cnt, part_ring;  // part_ring: partial-sum areas, reused every part_ring ops
    uint8_t* ws;
    int* counters;
    float* partials;
    int64_t part_stride;     // floats per ring area: T * 2 * M * 16
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
__device__ __forceinline__ int atom_acq_rel_add(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// activations that no op of the batch writes: read-only path; those that an
// earlier op of the batch produced: L2 (coherent within the launch)
__device__ __forceinline__ uint4 ld_x(const void* p, bool produced) {
    uint4 v;
    if (produced)
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    else
        asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Bounded wait on a shared-memory barrier phase.  False (and the abort flags
// raised) once kWaitNs pass, or when another warp has raised an abort flag.
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
        __nanosleep(64);
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

// SPFP2, one row of block s: codes c0..c3 are the nibbles of sA (low 16
// bits), c4..c7 those of sB; TH = [H, H | 0x80, 0, 0] and TL = [L, L, 0, 0]
// are the byte tables of the block's exponent (bf16 of +-2^(e-10) has biased
// exponent E = 117 + e: high byte sign | E >> 1, low byte (E & 1) << 7).
// Out: P[0..3] = bf16 pairs of columns (0,1) (2,3) (4,5) (6,7).
__device__ __forceinline__ void decode_spfp2_bf16(uint32_t sA, uint32_t sB, uint32_t TH, uint32_t TL, uint32_t* P) {
    const uint32_t hA = prmt(TH, 0u, sA), lA = prmt(TL, 0u, sA);
    const uint32_t hB = prmt(TH, 0u, sB), lB = prmt(TL, 0u, sB);
    P[0] = prmt(lA, hA, 0x5140u);
    P[1] = prmt(lA, hA, 0x7362u);
    P[2] = prmt(lB, hB, 0x5140u);
    P[3] = prmt(lB, hB, 0x7362u);
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
// tiles of 8; acc[0] / acc[1] take the two MMAs of a step.
template <int FMT, int NTB>
__device__ __forceinline__ void unit_mma(const uint32_t* fw, const uint16_t* const (&xr)[NTB], const bool (&xv)[NTB],
                                         int64_t col, bool produced, const uint32_t* pair_tab,
                                         const uint32_t* scale_tab, float (&acc)[2][NTB][4]) {
    // one token tile: the unit's activations for all 8 steps are loaded first,
    // so their latency overlaps the decode
    uint4 xs[NTB == 1 ? 8 : 1];
    if constexpr (NTB == 1) {
#pragma unroll
        for (int s = 0; s < 8; ++s) xs[s] = xv[0] ? ld_x(xr[0] + col + 8 * s, produced) : make_uint4(0u, 0u, 0u, 0u);
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
            const uint32_t W = fw[s];
            decode_spfp2_bf16(W & 0x3333u, (W >> 2) & 0x3333u, prmt(Hg, Hg | 0x80808080u, selH), prmt(Lg, 0u, selL),
                              A0);
            decode_spfp2_bf16((W >> 16) & 0x3333u, (W >> 18) & 0x3333u, prmt(Hh, Hh | 0x80808080u, selH),
                              prmt(Lh, 0u, selL), A1);
        } else {
            constexpr int CW = FMT == SPARK_FMT_FP3 ? 6 : 8;
            decode_scaled<FMT>(fw, fw[CW], s, pair_tab, scale_tab, A0);
            decode_scaled<FMT>(fw + CW + 1, fw[2 * CW + 1], s, pair_tab, scale_tab, A1);
        }
#pragma unroll
        for (int j = 0; j < NTB; ++j) {
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if constexpr (NTB == 1) x = xs[s];
            else if (xv[j]) x = ld_x(xr[j] + col + 8 * s, produced);
            mma_bf16(acc[0][j], A0[0], A1[0], A0[1], A1[1], x.x, x.y);
            mma_bf16(acc[1][j], A0[2], A1[2], A0[3], A1[3], x.z, x.w);
        }
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
    int* op_done;
};

// Row-group segments of op k are held as v[2j + i][r] = row g (r = 0) / g + 8
// (r = 1) of token 8j + 2t + i.  write_rows writes a whole row group;
// flush_partial publishes the partial of a segment, and the last contributor
// sums the partials in unit order and writes the rows.
template <int NV>
__device__ __forceinline__ void write_rows(const Op& op, int M, int rg, const float (&v)[NV][2], int lane) {
    const int g = lane >> 2, t = lane & 3;
    {
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
}

template <int NV>
__device__ __noinline__ void flush_partial(const Args& a, const Ctl& C, int k, int vw, int rg, int slot,
                                           const float (&v)[NV][2], int lane) {
    const Op& op = a.op[k];
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M;
    float* area = a.partials + (int64_t)(k % a.part_ring) * a.part_stride;
    // areas are reused every part_ring ops: the op that last used this one
    // must be finished (every warp past it, its partials read)
    if (k >= a.part_ring) {
        bool ok = true;
        if (lane == 0) ok = wait_count(C.op_done + (k - a.part_ring), gridDim.x * kCW, C.abort, C.err);
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
    __syncwarp();
    const int first = rg * op.n_kc;
    const int v_lo = vw_owner(op, first), v_hi = vw_owner(op, first + op.n_kc - 1);
    int old = 0;
    if (lane == 0) {
        __threadfence_block();
        old = atom_acq_rel_add(a.counters + op.cnt_off + rg, 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != v_hi - v_lo) return;
    // the first contributor holds this row group in its second slot when its
    // sub-range began in an earlier row group
    const int lo_slot = vw_start(op, v_lo) < first ? 1 : 0;
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
    if (lane == 0) a.counters[op.cnt_off + rg] = 0;
}

// ---------------------------------------------------------------- roles
__device__ void producer(const Args& a, uint8_t* ring, uint64_t* full, uint64_t* empty, const Ctl& C,
                         volatile int* s_abort) {
    const int G = gridDim.x, c = blockIdx.x;
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    uint32_t q = 0;
    bool stop = false;
    const uint32_t ring0 = smem_u32(ring);
    for (int k = 0; k < a.n_ops && !stop; ++k) {
        const Op& op = a.op[k];
        const int cr = (c + k) % G;
        const int S = op.q + (cr < op.rem ? 1 : 0);
        const uint32_t ub = (uint32_t)op.unit_bytes;
        // per consumer warp: its first unit's address; warps with v < rem hold
        // one unit more (the last stage's), the others q
        const uint8_t* src[kCW];
        int n_long = 0;
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
            const int v = ((w + k) % kCW) * G + cr;
            src[w] = op.w + (int64_t)vw_start(op, v) * ub;
            n_long += v < op.rem ? 1 : 0;
        }
        for (int s = 0; s < S; ++s, ++q) {
            const uint32_t st = q % kStages;
            if (!wait_phase(smem_u32(empty + st), ((q / kStages) & 1u) ^ 1u, s_abort, C.abort, C.err) || *C.abort) {
                *s_abort = 1;
                stop = true;
                break;
            }
            const bool last = s == op.q;
            const uint32_t fb = smem_u32(full + st);
            mbar_expect_tx(fb, (uint32_t)((last ? n_long : kCW) * op.unit_bytes));
            const uint32_t dst0 = ring0 + st * kStageBytes;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                // on the last stage only warps w' * G + c' < rem have a unit
                if (last && ((w + k) % kCW) * G + cr >= op.rem) continue;
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
                    "%2, [%3], %4;" ::"r"(dst0 + w * kSlotBytes),
                    "l"(src[w] + (int64_t)s * ub), "r"(ub), "r"(fb), "l"(policy)
                    : "memory");
            }
        }
    }
    if (stop) {
        // let the copies already issued land before the CTA retires
        const uint32_t lo = q > kStages ? q - kStages : 0;
        for (uint32_t p = lo; p < q; ++p) {
            const uint64_t dl = globaltimer_ns() + kWaitNs;
            while (!mbar_try(smem_u32(full + p % kStages), (p / kStages) & 1u) && globaltimer_ns() < dl) {
            }
        }
    }
}

template <int NTB>
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
        const bool produced = op.dep0 >= 0 || op.dep1 >= 0;
        if (mine > 0 && !dead && produced) {
            // earlier ops of the batch whose output this op reads
            bool ok = true;
            if (lane == 0) {
                if (op.dep0 >= 0) ok = wait_count(C.op_done + op.dep0, T, C.abort, C.err);
                if (ok && op.dep1 >= 0) ok = wait_count(C.op_done + op.dep1, T, C.abort, C.err);
            }
            dead = !__shfl_sync(0xffffffffu, ok ? 1 : 0, 0);
        }
        int kc = mine > 0 ? u0 % op.n_kc : 0, rg = mine > 0 ? u0 / op.n_kc : 0;
        const int rg_first = rg;
        int seg0 = u0;
        float acc[2][NTB][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < NTB; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[h][j][i] = 0.0f;
        const uint16_t* xr[NTB];
        bool xv[NTB];
#pragma unroll
        for (int j = 0; j < NTB; ++j) {
            xv[j] = 8 * j + g < M;
            xr[j] = op.x + (int64_t)(8 * j + g) * op.ldx;
        }
        for (int s = 0; s < S; ++s, ++q) {
            const uint32_t st = q % kStages;
            const bool have = s < mine;
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

            const int64_t col = (int64_t)kc * 256 + t * 64;
            if (op.fmt == SPARK_FMT_SPFP2)
                unit_mma<SPARK_FMT_SPFP2, NTB>(fw, xr, xv, col, produced, pair_fp3, scale_tab, acc);
            else if (op.fmt == SPARK_FMT_FP3)
                unit_mma<SPARK_FMT_FP3, NTB>(fw, xr, xv, col, produced, pair_fp3, scale_tab, acc);
            else
                unit_mma<SPARK_FMT_NVFP4, NTB>(fw, xr, xv, col, produced, pair_nv, scale_tab, acc);

            const int u = u0 + s;
            if (kc == op.n_kc - 1 || s + 1 == mine) {
                float vals[2 * NTB][2];
#pragma unroll
                for (int j = 0; j < NTB; ++j)
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        vals[2 * j + i][0] = acc[0][j][i] + acc[1][j][i];
                        vals[2 * j + i][1] = acc[0][j][2 + i] + acc[1][j][2 + i];
                    }
                if (seg0 == rg * op.n_kc && u + 1 == (rg + 1) * op.n_kc)
                    write_rows<2 * NTB>(op, M, rg, vals, lane);
                else
                    flush_partial<2 * NTB>(a, C, k, vw, rg, rg == rg_first ? 0 : 1, vals, lane);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int j = 0; j < NTB; ++j)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[h][j][i] = 0.0f;
                seg0 = u + 1;
            }
            if (++kc == op.n_kc) {
                kc = 0;
                ++rg;
            }
        }
        // this warp is done with op k (outputs and partial reads included); the
        // count is kept only for ops that something waits on
        if (op.waited) {
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                red_release_add(C.op_done + k, 1);
            }
        }
    }
}

template <int NTB>
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
    Ctl C;
    C.err = reinterpret_cast<int*>(a.ws);
    C.abort = reinterpret_cast<volatile int*>(a.ws + kCtlAbort);
    C.op_done = reinterpret_cast<int*>(a.ws + kCtlOpDone);
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
    } else {
        consumer<NTB>(a, ring, full, empty, C, sab, pair_fp3, pair_nv, scale_tab, warp, lane);
    }
    __syncthreads();
    // the last CTA out returns the control block to zero for the next launch
    if (threadIdx.x == 0) {
        __threadfence();
        const int old = atomicAdd(reinterpret_cast<int*>(a.ws + kCtlCtaDone), 1);
        if (old == (int)gridDim.x - 1) {
            __threadfence();
            for (int k = 0; k < a.n_ops; ++k) C.op_done[k] = 0;
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
static_assert(kSmemBytes <= 227 * 1024, "shared memory above the per-CTA limit");

int sm_count(int dev) {
    static int cache[64] = {};
    if (dev < 0 || dev >= 64) return 0;
    if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
    return cache[dev];
}

std::mutex g_mu;

template <int NTB>
int launch(const Args& a, int grid, cudaStream_t s) {
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
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
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
    int64_t cnt = 0;
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
    }
    a.n_cnt = (int)std::min<int64_t>(cnt, max_counters);
    SPARK_REQUIRE(cnt <= max_counters, SPARK_ERR_UNSUPPORTED,
                  "spark_linear_batch: %lld row groups in the batch, above %lld", (long long)cnt, (long long)max_counters);
    const int64_t T = (int64_t)G * kCW;
    a.part_stride = T * 2 * M * 16;
    const size_t area = (size_t)a.part_stride * sizeof(float);
    a.part_ring = (int)std::max<size_t>(1, std::min<size_t>((size_t)n_ops, kPartAreaBudget / area));
    for (int k = 0; k < n_ops; ++k) {
        Op& p = a.op[k];
        if (k + a.part_ring < n_ops) p.waited = 1;
        if (p.dep0 >= 0) a.op[p.dep0].waited = 1;
        if (p.dep1 >= 0) a.op[p.dep1].waited = 1;
    }
    P->scratch_bytes = ((size_t)a.part_ring * area + 255) / 256 * 256;
    P->grid = G;
    a.ws = ws;
    if (ws) {
        a.counters = reinterpret_cast<int*>(ws + counters_off);
        a.partials = reinterpret_cast<float*>(ws + scratch_off);
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
    (void)ic;
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t Mc = M < 1 ? 1 : (M > stream::kMaxTok ? stream::kMaxTok : M);
    const size_t part = (size_t)stream::sm_count(dev) * stream::kCW * 2 * Mc * 16 * sizeof(float);
    return (part + 255) / 256 * 256;
}

int stream_launch(const StreamPlan& P, cudaStream_t s) {
    const stream::Args& a = P.args;
    return a.M <= 8 ? stream::launch<1>(a, P.grid, s) : stream::launch<2>(a, P.grid, s);
}

}  // namespace spark
