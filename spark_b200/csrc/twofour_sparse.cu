// twofour_sparse.cu -- 2:4-sparse SPFP2 linear on the sparse tensor cores.
//
// y[M, oc] = x[M, ic] . decode(W)^T (+ bias) with W in the reference's 2:4
// layout (two_four.py:112-155: per 16 weights a 28-bit field, 7 bytes per
// pair of fields; four groups of four columns, each with a 4-bit mode --
// the two nonzero positions (modes 0-5), one (8-11) or none -- two sign
// bits and a shared 4-bit exponent: a nonzero is +-2^(e - 10)).  Each group
// holds at most two nonzeros, which is the 2:4 structure the sparse MMA
// takes: tcgen05.mma.sp kind::f16 multiplies the compressed weights (the two
// kept values of every group, bf16, exact) by the caller's bf16 x, with the
// positions as 2-bit metadata indices, so half the MMA work of the dense
// decode is skipped.
//
// Tile: 128 weight rows x 128 tokens per CTA; K in blocks of 128 columns.
// Roles (32 * (4 * kGroups + 2) threads):
//   warps 0 .. 4*kGroups-1  decoders, then the epilogue.  kGroups groups of
//              four warps decode alternate K blocks (group g the blocks
//              kb = g mod kGroups), warp w for the 32 weight rows of lane
//              quadrant w % 4; its thread r decodes row r of the block: the
//              64 kept values of its 32 groups go to
//              the block's A stage in shared memory (one 128-byte-swizzled,
//              K-major row, the MMA's compressed operand), the group indices
//              to the block's metadata columns in TMEM: per MMA (32 columns)
//              one 32-bit column, lane 16*(m/16) + 8*(k/16) + m%8 holding bit
//              k%16 + 16*((m/8)%2) of row m (each group's nibble: first index
//              in bits 0-1, second in bits 2-3, first < second).  Rows reach
//              their lanes by two warp shuffles per MMA.
//   next warp  lane 0 issues the TMA loads of the activation tiles.
//   last warp  allocates TMEM; lane 0 issues 4 sparse MMAs per block and
//              commits each block back to its producers.
// Every wait is bounded (2 s): an expired wait stores error code 6 in the
// caller's error word, and every role still reaches the final barrier and
// frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "tc_common.cuh"

namespace spark {
namespace tc {
int get_encoder();
int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);
}  // namespace tc

namespace tfs {
using namespace tcx;

constexpr int kRows = 128, kTok = 128, kKB = 128;     // K columns per block
constexpr int kStages = 4;
constexpr int kStageA = kRows * 128;                  // 64 kept bf16 values per row
constexpr int kStageB = kTok * kKB * 2;               // two 64-column swizzled boxes
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kSmem = kStages * kStageBytes + 1024;
// One decoder warp per lane quadrant handles a block alone, and its chain per
// block (loads, table lookups, shared and TMEM stores, fences) is what bounds
// the kernel, so groups of four warps take alternate blocks.
constexpr int kGroups = 3;
constexpr int kDecWarps = 4 * kGroups;
constexpr int kThreads = 32 * (kDecWarps + 2);
constexpr int kTmaWarp = kDecWarps, kMmaWarp = kDecWarps + 1;
constexpr uint32_t kTmemCols = 256;                   // D: 128 columns; metadata: 4 per stage
constexpr uint32_t kECol = 128;
// bf16 x bf16 -> f32, K-major, N = kTok, M = 128, sparse (bit 2)
constexpr uint32_t kIdesc =
    (1u << 2) | (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTok >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

__device__ __forceinline__ void mma_sp(uint32_t d, uint64_t a, uint64_t b, uint32_t e, uint32_t acc) {
    // the metadata address carries its column-pair selector in bit 0 (the
    // instruction descriptor's sparse id2 field); the address itself is even
    const uint32_t idesc = kIdesc | (e & 1u);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%9], %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(e & ~1u)
        : "memory");
}
__device__ __forceinline__ void tmem_st2(uint32_t taddr, uint32_t a, uint32_t b) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(a), "r"(b) : "memory");
}

struct Params {
    const uint8_t* wq;      // 2:4 rows, ic * 7 / 32 bytes each
    const void* bias;
    void* y;
    int64_t ldy, row_bytes;
    int M, oc, n_kb, bias_dtype, y_dtype;
    int split;              // K ranges (blockIdx.z); above 1: fp32 partials and a last-CTA sum
    float* part;            // [split][M][oc] partial sums (split > 1): a warp's 32 rows are contiguous
    int* cnt;               // per output tile: CTAs done, back to zero after the sum (split > 1)
    int* err;
};

// Per (mode, s0, s1) of a group: the metadata nibble (bits 0-3), then which of
// the two kept slots hold a nonzero and its sign (bits 8-11).
__device__ __forceinline__ uint32_t group_entry(uint32_t idx) {
    const uint32_t mode = idx & 15u, s0 = (idx >> 4) & 1u, s1 = (idx >> 5) & 1u;
    const uint32_t pa[6] = {0, 0, 0, 1, 1, 2}, pb[6] = {1, 2, 3, 2, 3, 3};
    if (mode < 6) return pa[mode] | (pb[mode] << 2) | (1u << 8) | (s0 << 9) | (1u << 10) | (s1 << 11);
    if (mode >= 8 && mode <= 11) {
        const uint32_t p = mode - 8;
        // one nonzero at p: pair it with column 3 (a zero), or with 2 when p is 3
        return p < 3 ? (p | (3u << 2) | (1u << 8) | (s0 << 9)) : (2u | (3u << 2) | (1u << 10) | (s0 << 11));
    }
    return 0u | (1u << 2);   // no nonzero: columns 0 and 1, both zero
}

__global__ void __launch_bounds__(kThreads, 1)
    k_twofour_sparse(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[3 * kStages + 1];
    __shared__ uint32_t s_tmem;
    __shared__ uint16_t s_tab[64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kRows, tok0 = blockIdx.y * kTok;
    // this CTA's K blocks [kb0, kb0 + nk); blocks below are numbered from kb0
    const int kb0 = (int)((int64_t)blockIdx.z * p.n_kb / p.split);
    const int nk = (int)((int64_t)(blockIdx.z + 1) * p.n_kb / p.split) - kb0;
    __shared__ int s_last;
    const uint32_t bfull = smem_u32(&bars[0]), empty = smem_u32(&bars[kStages]), afull = smem_u32(&bars[2 * kStages]);
    const uint32_t done = smem_u32(&bars[3 * kStages]);
    if (threadIdx.x < 64) s_tab[threadIdx.x] = (uint16_t)group_entry(threadIdx.x);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bfull + 8 * s, 1);
            mbar_init(empty + 8 * s, 1);
            mbar_init(afull + 8 * s, 4);   // the four warps of the block's group
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = s_tmem;
    bool ok = true;

    if (warp == kTmaWarp) {
        if (lane == 0) {
            for (int kb = 0; kb < nk && ok; ++kb) {
                const int s = kb % kStages;
                if (kb >= kStages) ok = mbar_wait(empty + 8 * s, (uint32_t)((kb / kStages - 1) & 1));
                if (!ok) break;
                const uint32_t st = smem_u32(smem + s * kStageBytes + kStageA);
                mbar_expect_tx(bfull + 8 * s, kStageB);
                tma_load_2d(st, &xmap, (kb0 + kb) * kKB, tok0, bfull + 8 * s);
                tma_load_2d(st + kStageB / 2, &xmap, (kb0 + kb) * kKB + 64, tok0, bfull + 8 * s);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (int kb = 0; kb < nk && ok; ++kb) {
                const int s = kb % kStages;
                const uint32_t par = (uint32_t)((kb / kStages) & 1);
                ok = mbar_wait(bfull + 8 * s, par) && mbar_wait(afull + 8 * s, par);
                if (!ok) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * kStageBytes), sb = sa + kStageA;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_sp(tbase, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + (kk >> 1) * (kStageB / 2) + (kk & 1) * 64),
                           tbase + kECol + (uint32_t)(s * 4 + kk), (kb | kk) != 0);
                mma_commit(empty + 8 * s);
            }
            mma_commit(done);
        }
    } else {
        const int q = warp & 3, grp = warp >> 2, r = q * 32 + lane;   // weight row in the tile, decoder group
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const uint32_t* wrow = reinterpret_cast<const uint32_t*>(p.wq + (int64_t)(row0 + r) * p.row_bytes);
        // the two rows whose metadata halves this lane's TMEM word holds
        const int lm1 = 16 * (lane >> 4) + (lane & 7), hsel = (lane >> 3) & 1;
        // the row's 28 bytes of this group's next block, loaded one block ahead
        uint32_t wn[7] = {0u, 0u, 0u, 0u, 0u, 0u, 0u};
        if (grp < nk) {
#pragma unroll
            for (int i = 0; i < 7; ++i) wn[i] = wrow[7 * (kb0 + grp) + i];
        }
        for (int kb = grp; kb < nk && ok; kb += kGroups) {
            const int s = kb % kStages;
            if (kb >= kStages) ok = mbar_wait(empty + 8 * s, (uint32_t)((kb / kStages - 1) & 1));
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            // 128 columns = 8 fields = 28 bytes of the row
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 7; ++i) w[i] = wn[i];
            w[7] = 0u;
            if (kb + kGroups < nk) {
#pragma unroll
                for (int i = 0; i < 7; ++i) wn[i] = wrow[7 * (kb0 + kb + kGroups) + i];
            }
            uint32_t kept[32], meta[4];
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) {
                const int bit = 56 * pp, wi = bit >> 5, off = bit & 31;
                const uint32_t lo = off ? __funnelshift_r(w[wi], w[wi + 1], off) : w[wi];
                const uint32_t hi = off ? __funnelshift_r(w[wi + 1], w[wi + 2], off) : w[wi + 1];
                uint32_t m32 = 0u;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t f = h ? (__funnelshift_r(lo, hi, 28) & 0x0fffffffu) : (lo & 0x0fffffffu);
                    const uint32_t mag = (117u + ((f >> 24) & 15u)) << 7;   // bf16 bits of 2^(e - 10)
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint32_t t = s_tab[((f >> (4 * g)) & 15u) | (((f >> (16 + 2 * g)) & 3u) << 4)];
                        const uint32_t v0 = (t & 0x100u) ? (mag | ((t >> 9) & 1u) << 15) : 0u;
                        const uint32_t v1 = (t & 0x400u) ? (mag | ((t >> 11) & 1u) << 15) : 0u;
                        kept[(2 * pp + h) * 4 + g] = v0 | (v1 << 16);
                        m32 |= (t & 15u) << (16 * h + 4 * g);
                    }
                }
                meta[pp] = m32;                                  // MMA pp: columns 32pp .. 32pp + 31
            }
            // kept values: this row of the A stage, 16-byte chunks swizzled by row
            uint8_t* arow = smem + s * kStageBytes + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) =
                    make_uint4(kept[4 * c], kept[4 * c + 1], kept[4 * c + 2], kept[4 * c + 3]);
            // metadata: lane l takes half hsel of rows lm1 and lm1 + 8 of this warp
            uint32_t ev[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t a = __shfl_sync(0xffffffffu, meta[kk], lm1);
                const uint32_t b = __shfl_sync(0xffffffffu, meta[kk], lm1 + 8);
                ev[kk] = (hsel ? (a >> 16) : (a & 0xffffu)) | ((hsel ? (b >> 16) : (b & 0xffffu)) << 16);
            }
            tmem_st2(tbase + lane_off + kECol + (uint32_t)(s * 4), ev[0], ev[1]);
            tmem_st2(tbase + lane_off + kECol + (uint32_t)(s * 4 + 2), ev[2], ev[3]);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the A stage, for the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull + 8 * s);
        }
        // epilogue: this quadrant's 32 weight rows, the groups taking 16-column chunks in turn
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(done, 0));
        const int64_t row = row0 + r;
        const float b = p.bias ? load_as_float(p.bias, p.bias_dtype, row) : 0.0f;
        if (p.split == 1) {
            if (ok) {
                tc_fence_after();
                for (int c0 = 16 * grp; c0 < kTok; c0 += 16 * kGroups) {
                    float v[16];
                    tmem_ld16(tbase + lane_off + (uint32_t)c0, v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int t = tok0 + c0 + i;
                        if (t < p.M) store_from_float(p.y, p.y_dtype, (int64_t)t * p.ldy + row, v[i] + b);
                    }
                }
            }
        } else {
            // K split: store this range's fp32 sums; the CTA that completes the
            // tile's count adds the ranges in order 0..split-1 (the result does
            // not depend on which CTA finishes last) and writes y.  Every decoder
            // thread passes both barriers, also after an error.
            float* mine = p.part + (int64_t)blockIdx.z * p.oc * p.M;
            if (ok) {
                tc_fence_after();
                for (int c0 = 16 * grp; c0 < kTok && tok0 + c0 < p.M; c0 += 16 * kGroups) {
                    float v[16];
                    tmem_ld16(tbase + lane_off + (uint32_t)c0, v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int t = tok0 + c0 + i;
                        if (t < p.M) __stcg(mine + (int64_t)t * p.oc + row, v[i]);
                    }
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"r"(kDecWarps * 32) : "memory");
            int* cnt = p.cnt + blockIdx.y * gridDim.x + blockIdx.x;
            if (threadIdx.x == 0) s_last = atomicAdd(cnt, 1) == p.split - 1;
            asm volatile("bar.sync 1, %0;" ::"r"(kDecWarps * 32) : "memory");
            if (s_last) {
                __threadfence();
                for (int c = grp; c < kTok && tok0 + c < p.M; c += kGroups) {
                    const int t = tok0 + c;
                    float sum = 0.0f;
                    for (int z = 0; z < p.split; ++z) sum += __ldcg(p.part + ((int64_t)z * p.M + t) * p.oc + row);
                    store_from_float(p.y, p.y_dtype, (int64_t)t * p.ldy + row, sum + b);
                }
                if (threadIdx.x == 0) *cnt = 0;
            }
        }
    }
    if (!ok) report_device_error(p.err, 6);
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols) : "memory");
    }
}

}  // namespace tfs

// counters (int[], zero, left zero) and part (part_bytes) : scratch for the
// K split of small token counts; null counters: no split.
int twofour_sparse_run(const uint8_t* wq, const void* x, int64_t M, int64_t oc, int64_t ic, const void* bias,
                       int bias_dtype, void* y, int y_dtype, int64_t ldy, int* err, int* counters, float* part,
                       size_t part_bytes, cudaStream_t stream) {
    using namespace spark::tfs;
    SPARK_REQUIRE(wq && x && y && err, SPARK_ERR_INVALID, "spark_twofour_sparse_linear: null pointer");
    SPARK_REQUIRE(M >= 1 && M < (1ll << 31) && oc >= kRows && oc % kRows == 0 && oc < (1ll << 31) && ic >= kKB &&
                      ic % kKB == 0 && ic < (1ll << 31),
                  SPARK_ERR_INVALID,
                  "spark_twofour_sparse_linear: oc a multiple of %d, ic a multiple of %d (got %lld, %lld)", kRows, kKB,
                  (long long)oc, (long long)ic);
    SPARK_REQUIRE(y_dtype >= 0 && y_dtype <= 2 && ldy >= oc && (!bias || (bias_dtype >= 0 && bias_dtype <= 2)),
                  SPARK_ERR_INVALID, "spark_twofour_sparse_linear: y / bias");
    SPARK_REQUIRE(aligned(wq, 4) && aligned(x, 16), SPARK_ERR_ALIGNMENT,
                  "spark_twofour_sparse_linear: 4-byte aligned weights, 16-byte aligned x");
    int rc = tc::get_encoder();
    if (rc) return rc;
    CUtensorMap xmap;
    rc = tc::encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)ic, (uint64_t)M, (uint64_t)ic * 2, 64,
                       kTok, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    cudaError_t e = cudaFuncSetAttribute(k_twofour_sparse, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return set_error((int)e, "spark_twofour_sparse_linear: %s", cudaGetErrorString(e));
    Params p;
    p.wq = wq;
    p.bias = bias;
    p.y = y;
    p.ldy = ldy;
    p.row_bytes = ic / 32 * 7;
    p.M = (int)M;
    p.oc = (int)oc;
    p.n_kb = (int)(ic / kKB);
    p.bias_dtype = bias_dtype;
    p.y_dtype = y_dtype;
    p.err = err;
    p.split = 1;
    p.part = nullptr;
    p.cnt = nullptr;
    // few output tiles (decode sizes): split K so that about one CTA per SM
    // runs; the ranges' fp32 sums go to the caller's scratch
    const int64_t tiles = (oc / kRows) * ((M + kTok - 1) / kTok);
    if (counters && part && tiles < 74) {
        int sm = 0, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
        int64_t split = std::min<int64_t>({(int64_t)sm / tiles, (int64_t)p.n_kb, (int64_t)16});
        while (split > 1 && (size_t)split * oc * M * sizeof(float) > part_bytes) --split;
        if (split > 1) {
            p.split = (int)split;
            p.cnt = counters;
            p.part = part;
        }
    }
    const dim3 grid((unsigned)(oc / kRows), (unsigned)((M + kTok - 1) / kTok), (unsigned)p.split);
    k_twofour_sparse<<<grid, kThreads, kSmem, stream>>>(xmap, p);
    return check_launch("spark_twofour_sparse_linear");
}

}  // namespace spark

extern "C" {

int spark_twofour_sparse_linear(const uint8_t* wq, const void* x, int64_t M, int64_t oc, int64_t ic, const void* bias,
                                int bias_dtype, void* y, int y_dtype, int64_t ldy, int* err, void* stream) {
    return spark::twofour_sparse_run(wq, x, M, oc, ic, bias, bias_dtype, y, y_dtype, ldy, err, nullptr, nullptr, 0,
                                     reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
