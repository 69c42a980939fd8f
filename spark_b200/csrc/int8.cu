// int8.cu -- per-output-channel symmetric INT8 (01_core/int8_emu.py), the
// lm_head tier of the reference's mixed quantisation:
//   scale_r = max(amax|w_r| / 127, 1e-12)              (int8_emu.py:15, :43)
//   q       = clamp(round_half_even(w / scale_r), +-127) (:16, :44)
//   fake    = q * scale_r                               (:17)
// One CTA per row: a max-reduction over the row, then one pass that writes q
// (int8) or q * scale.  fp32 arithmetic with the reference's operation order;
// a NaN anywhere in a row makes its scale NaN, as torch's amax does.
#include "common.cuh"

namespace spark {
namespace {

constexpr int kRowThreads = 256;

// max of |w| over the row as raw bits: for non-negative floats the integer
// order is the float order, and every NaN compares above +inf
__device__ float row_scale(const void* w, int dtype, int64_t row, int64_t ic, uint32_t* red) {
    uint32_t m = 0;
    for (int64_t c = threadIdx.x; c < ic; c += blockDim.x)
        m = max(m, __float_as_uint(load_as_float(w, dtype, row * ic + c)) & 0x7fffffffu);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float amax = __uint_as_float(red[0] > 0x7f800000u ? 0x7fc00000u : red[0]);
    const float s = __fdiv_rn(amax, 127.0f);
    return s < 1e-12f ? 1e-12f : s;     // a NaN scale stays NaN
}

__device__ __forceinline__ float quantize(float v, float s) {
    float q = rintf(__fdiv_rn(v, s));
    return q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
}

__global__ void __launch_bounds__(kRowThreads) k_int8_fake_quant(const void* __restrict__ w, int dtype, int64_t ic,
                                                                  void* __restrict__ out, int out_dtype) {
    __shared__ uint32_t red[32];
    const int64_t row = blockIdx.x;
    const float s = row_scale(w, dtype, row, ic, red);
    for (int64_t c = threadIdx.x; c < ic; c += blockDim.x) {
        const int64_t i = row * ic + c;
        store_from_float(out, out_dtype, i, __fmul_rn(quantize(load_as_float(w, dtype, i), s), s));
    }
}

__global__ void __launch_bounds__(kRowThreads) k_int8_pack(const void* __restrict__ w, int dtype, int64_t ic,
                                                            int8_t* __restrict__ q, float* __restrict__ scale) {
    __shared__ uint32_t red[32];
    const int64_t row = blockIdx.x;
    const float s = row_scale(w, dtype, row, ic, red);
    if (threadIdx.x == 0) scale[row] = s;
    for (int64_t c = threadIdx.x; c < ic; c += blockDim.x) {
        const int64_t i = row * ic + c;
        q[i] = (int8_t)(int)quantize(load_as_float(w, dtype, i), s);
    }
}

__global__ void k_int8_unpack(const int8_t* __restrict__ q, const float* __restrict__ scale, int64_t oc, int64_t ic,
                              void* __restrict__ out, int out_dtype) {
    const int64_t n = oc * ic;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_from_float(out, out_dtype, i, __fmul_rn((float)q[i], scale[i / ic]));
}

bool dtype_valid(int d) { return d == SPARK_DTYPE_F32 || d == SPARK_DTYPE_BF16 || d == SPARK_DTYPE_F16; }

}  // namespace
}  // namespace spark

using namespace spark;

extern "C" {

int spark_int8_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype,
                          void* stream) {
    SPARK_REQUIRE(w && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_int8_fake_quant: null pointer");
    SPARK_REQUIRE(dtype_valid(w_dtype) && dtype_valid(out_dtype), SPARK_ERR_INVALID, "spark_int8_fake_quant: bad dtype");
    SPARK_REQUIRE(oc < (1ll << 31), SPARK_ERR_UNSUPPORTED, "spark_int8_fake_quant: too many rows");
    if (oc == 0 || ic == 0) return SPARK_OK;
    k_int8_fake_quant<<<(unsigned)oc, kRowThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, w_dtype, ic, out,
                                                                                                 out_dtype);
    return check_launch("spark_int8_fake_quant");
}

int spark_int8_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, int8_t* q, float* scale, void* stream) {
    SPARK_REQUIRE(w && q && scale && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_int8_pack: null pointer");
    SPARK_REQUIRE(dtype_valid(w_dtype), SPARK_ERR_INVALID, "spark_int8_pack: bad dtype %d", w_dtype);
    SPARK_REQUIRE(oc < (1ll << 31), SPARK_ERR_UNSUPPORTED, "spark_int8_pack: too many rows");
    if (oc == 0 || ic == 0) return SPARK_OK;
    k_int8_pack<<<(unsigned)oc, kRowThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, w_dtype, ic, q, scale);
    return check_launch("spark_int8_pack");
}

int spark_int8_unpack(const int8_t* q, const float* scale, int64_t oc, int64_t ic, void* out, int out_dtype,
                      void* stream) {
    SPARK_REQUIRE(q && scale && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_int8_unpack: null pointer");
    SPARK_REQUIRE(dtype_valid(out_dtype), SPARK_ERR_INVALID, "spark_int8_unpack: bad dtype %d", out_dtype);
    if (oc == 0 || ic == 0) return SPARK_OK;
    const int64_t n = oc * ic;
    const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
    k_int8_unpack<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(q, scale, oc, ic, out, out_dtype);
    return check_launch("spark_int8_unpack");
}

}  // extern "C"
