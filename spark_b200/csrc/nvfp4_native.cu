// nvfp4_native.cu -- NVFP4 x NVFP4 on the block-scaled FP4 tensor cores.
//
// A reported mode beside the parity path: the activations are quantised to
// NVFP4 too (the reference's per-16 quantiser, nvfp4_emu.py:37-57, applied to
// x by spark_nvfp4_pack), and y[M, oc] = dequant(xq) . dequant(Wq)^T runs on
// tcgen05.mma kind::mxf4nvf4 with block16 (ue4m3) scales and fp32
// accumulation: both operands stay packed (two e2m1 codes per byte, even
// element in the low nibble) and the scales are applied by the MMA.  The
// parity path (spark_linear: bf16 x times the exactly decoded weights) is
// unchanged; this mode trades the activations' FP4 rounding for 4x the MMA
// rate of bf16.
//
// Tile: 128 weight rows x 128 tokens per CTA, K in blocks of 256 (128 bytes
// of codes per row: one 128-byte-swizzled TMA box; 16 bytes of scales per
// row: one plain box), kStages blocks in flight, two CTAs per SM.
// Roles (192 threads):
//   warps 0-3  scale writers, then the epilogue: warp q owns TMEM lanes
//              32q..32q+31.  Per K block each thread reads the 16 scale
//              bytes of weight rows g*32 + l and of tokens g*32 + l (g = 0..3)
//              from the stage and stores them with tcgen05.st into the
//              block's scale columns: per MMA (K = 64) column g holds the 4
//              scales of rows g*32 + lane in one 32-bit word, replicated in
//              all four lane quadrants (the layout the block-scaled MMA reads).
//   warp 4     lane 0 issues the TMA loads of the code and scale tiles.
//   warp 5     allocates TMEM; lane 0 issues the MMAs (4 per K block) and
//              commits each block back to its producers.
// Every mbarrier wait is bounded (2 s); an expired wait records error code 4
// in the caller's error word and every role still reaches the final barrier
// and frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace spark {
namespace tc {
int get_encoder();
int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw);
}  // namespace tc

namespace nvn {
using namespace tcx;

constexpr int kRows = 128;          // weight rows per CTA (MMA M)
constexpr int kTok = 128;           // tokens per CTA (MMA N)
constexpr int kKB = 256;            // K elements per block: 128 bytes of codes per row
constexpr int kStages = 3;
constexpr int kStageA = kRows * 128;
constexpr int kStageB = kTok * 128;
constexpr int kStageSA = kRows * 16, kStageSB = kTok * 16;  // scale tiles
constexpr int kStageBytes = kStageA + kStageB + kStageSA + kStageSB;
constexpr int kSmem = kStages * kStageBytes + 1024;          // + alignment slack
static_assert(2 * (kSmem + 256) <= 228 * 1024, "two CTAs per SM");
constexpr int kThreads = 192;
constexpr int kTmaWarp = 4, kMmaWarp = 5;
constexpr uint32_t kTmemCols = 256;                          // D: 128 columns; scales: 32 per stage
constexpr uint32_t kSfCol = 128;

// Block-scaled instruction descriptor: A and B e2m1 (bits 7-9, 10-12 = 1),
// K-major, N = kTok (bits 17-22: N >> 3), ue4m3 scales (bit 23 = 0),
// M = 128 (bits 24-28: M >> 4), scale byte ids 0, K = 64.
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | ((uint32_t)(kTok >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

__device__ __forceinline__ void mma_fp4(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(kIdesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
struct Params {
    void* y;
    int64_t ldy;
    int M, oc, n_kb, y_dtype;
    int* err;
};

__global__ void __launch_bounds__(kThreads, 2)
    k_nvfp4_native(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap wsmap, const __grid_constant__ CUtensorMap xsmap,
                   const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[3 * kStages + 1];
    __shared__ uint32_t s_tmem;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kRows, tok0 = blockIdx.y * kTok;
    const uint32_t full = smem_u32(&bars[0]), empty = smem_u32(&bars[kStages]), sfull = smem_u32(&bars[2 * kStages]);
    const uint32_t done = smem_u32(&bars[3 * kStages]);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + 8 * s, 1);
            mbar_init(empty + 8 * s, 1);
            mbar_init(sfull + 8 * s, 4);
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
            for (int kb = 0; kb < p.n_kb && ok; ++kb) {
                const int s = kb % kStages;
                if (kb >= kStages) ok = mbar_wait(empty + 8 * s, (uint32_t)((kb / kStages - 1) & 1));
                if (!ok) break;
                const uint32_t st = smem_u32(smem + s * kStageBytes);
                mbar_expect_tx(full + 8 * s, kStageBytes);
                tma_load_2d(st, &wmap, kb * 128, row0, full + 8 * s);
                tma_load_2d(st + kStageA, &xmap, kb * 128, tok0, full + 8 * s);
                tma_load_2d(st + kStageA + kStageB, &wsmap, kb * 16, row0, full + 8 * s);
                tma_load_2d(st + kStageA + kStageB + kStageSA, &xsmap, kb * 16, tok0, full + 8 * s);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (int kb = 0; kb < p.n_kb && ok; ++kb) {
                const int s = kb % kStages;
                const uint32_t par = (uint32_t)((kb / kStages) & 1);
                ok = mbar_wait(full + 8 * s, par) && mbar_wait(sfull + 8 * s, par);
                if (!ok) break;
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * kStageBytes);
                const uint32_t sf = tbase + kSfCol + (uint32_t)s * 32;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_fp4(tbase, sdesc_sw128(st + kk * 32), sdesc_sw128(st + kStageA + kk * 32), sf + kk * 4,
                            sf + 16 + kk * 4, (kb | kk) != 0);
                mma_commit(empty + 8 * s);
            }
            mma_commit(done);
        }
    } else {
        // scale writers: warp q writes its lane quadrant of every block's scale columns
        // (the stage's TMA waited for the MMAs of its previous block, so its
        // scale columns are free once the stage is full)
        const int q = warp;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        for (int kb = 0; kb < p.n_kb && ok; ++kb) {
            const int s = kb % kStages;
            ok = mbar_wait(full + 8 * s, (uint32_t)((kb / kStages) & 1));
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            const uint4* sa = reinterpret_cast<const uint4*>(smem + s * kStageBytes + kStageA + kStageB);
            const uint4* sb = sa + kRows;
            uint32_t va[16], vb[16];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint4 a = sa[g * 32 + lane], b = sb[g * 32 + lane];   // rows / tokens past the end read 0
                // word kk of a row's 16 scale bytes: its 4 scales of MMA kk
                va[0 * 4 + g] = a.x, va[1 * 4 + g] = a.y, va[2 * 4 + g] = a.z, va[3 * 4 + g] = a.w;
                vb[0 * 4 + g] = b.x, vb[1 * 4 + g] = b.y, vb[2 * 4 + g] = b.z, vb[3 * 4 + g] = b.w;
            }
            const uint32_t sf = tbase + lane_off + kSfCol + (uint32_t)s * 32;
            tmem_st16(sf, va);
            tmem_st16(sf + 16, vb);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sfull + 8 * s);
        }
        // epilogue: this quadrant's 32 weight rows, every token of the tile
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(done, 0));
        if (ok) {
            tc_fence_after();
            const int r = row0 + q * 32 + lane;
            for (int c0 = 0; c0 < kTok; c0 += 16) {
                float v[16];
                tmem_ld16(tbase + lane_off + (uint32_t)c0, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int t = tok0 + c0 + i;
                    if (t < p.M && r < p.oc) store_from_float(p.y, p.y_dtype, (int64_t)t * p.ldy + r, v[i]);
                }
            }
        }
    }
    if (!ok) report_device_error(p.err, 4);
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols) : "memory");
    }
}

}  // namespace nvn
}  // namespace spark

extern "C" {

int spark_nvfp4_native_linear(const uint8_t* wq, const uint8_t* w_scales, const uint8_t* xq, const uint8_t* x_scales,
                              int64_t M, int64_t oc, int64_t ic, void* y, int y_dtype, int64_t ldy, int* err,
                              void* stream) {
    using namespace spark;
    using namespace spark::nvn;
    SPARK_REQUIRE(wq && w_scales && xq && x_scales && y && err, SPARK_ERR_INVALID,
                  "spark_nvfp4_native_linear: null pointer");
    SPARK_REQUIRE(M >= 1 && M < (1ll << 31) && oc >= 1 && oc % kRows == 0 && oc < (1ll << 31) && ic >= kKB &&
                      ic % kKB == 0 && ic < (1ll << 31),
                  SPARK_ERR_INVALID, "spark_nvfp4_native_linear: oc a multiple of %d, ic a multiple of %d (got %lld, %lld)",
                  kRows, kKB, (long long)oc, (long long)ic);
    SPARK_REQUIRE(y_dtype >= 0 && y_dtype <= 2 && ldy >= oc, SPARK_ERR_INVALID, "spark_nvfp4_native_linear: y");
    SPARK_REQUIRE(aligned(wq, 16) && aligned(xq, 16) && aligned(w_scales, 16) && aligned(x_scales, 16),
                  SPARK_ERR_ALIGNMENT, "spark_nvfp4_native_linear: 16-byte aligned codes and scales");
    int rc = tc::get_encoder();
    if (rc) return rc;
    CUtensorMap wmap, xmap, wsmap, xsmap;
    rc = tc::encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)(ic / 2), (uint64_t)oc, (uint64_t)(ic / 2),
                       128, kRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tc::encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)(ic / 2), (uint64_t)M, (uint64_t)(ic / 2),
                       128, kTok, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // scales: [rows][ic / 16] bytes, e4m3 (non-negative, read as ue4m3)
    rc = tc::encode_2d(&wsmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_scales, (uint64_t)(ic / 16), (uint64_t)oc,
                       (uint64_t)(ic / 16), 16, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = tc::encode_2d(&xsmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, x_scales, (uint64_t)(ic / 16), (uint64_t)M,
                       (uint64_t)(ic / 16), 16, kTok, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    cudaError_t e = cudaFuncSetAttribute(k_nvfp4_native, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return set_error((int)e, "spark_nvfp4_native_linear: %s", cudaGetErrorString(e));
    Params p;
    p.y = y;
    p.ldy = ldy;
    p.M = (int)M;
    p.oc = (int)oc;
    p.n_kb = (int)(ic / kKB);
    p.y_dtype = y_dtype;
    p.err = err;
    const dim3 grid((unsigned)(oc / kRows), (unsigned)((M + kTok - 1) / kTok));
    k_nvfp4_native<<<grid, kThreads, kSmem, reinterpret_cast<cudaStream_t>(stream)>>>(wmap, xmap, wsmap, xsmap, p);
    return check_launch("spark_nvfp4_native_linear");
}

}  // extern "C"
