// api.cu -- error reporting and small utilities of the C ABI.
#include <stdarg.h>

#include <algorithm>
#include <stdio.h>

#include "common.cuh"

namespace spark {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error((int)e, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return SPARK_OK;
}

// SiLU(gate) * up, the MLP activation between gate/up and down projections.
template <typename T>
__global__ void k_silu_mul(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < n; i += stride) {
        float a = (float)g[i];
        float b = (float)u[i];
        o[i] = (T)(a / (1.0f + __expf(-a)) * b);
    }
}

// Row-strided form: gate / up rows `ld_in` elements apart (e.g. the two halves
// of a row-merged gate|up output), out rows `ld_out` apart.
template <typename T>
__global__ void k_silu_mul_rows(const T* __restrict__ g, const T* __restrict__ u, int64_t ld_in, T* __restrict__ o,
                                int64_t ld_out, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < n; i += stride) {
        const int64_t r = i / cols, c = i - r * cols;
        const float a = (float)g[r * ld_in + c];
        const float b = (float)u[r * ld_in + c];
        o[r * ld_out + c] = (T)(a / (1.0f + __expf(-a)) * b);
    }
}

}  // namespace spark

using namespace spark;

extern "C" {

const char* spark_last_error(void) { return g_last_error; }

int spark_version(void) { return 100; }

int spark_silu_mul(const void* gate, const void* up, void* out, int dtype, int64_t n, void* stream) {
    SPARK_REQUIRE(gate && up && out && n >= 0, SPARK_ERR_INVALID, "spark_silu_mul: null pointer");
    if (n == 0) return SPARK_OK;
    int grid = (int)((n + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SPARK_DTYPE_F32)
        k_silu_mul<float><<<grid, 256, 0, s>>>((const float*)gate, (const float*)up, (float*)out, n);
    else if (dtype == SPARK_DTYPE_BF16)
        k_silu_mul<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)gate, (const __nv_bfloat16*)up,
                                                       (__nv_bfloat16*)out, n);
    else if (dtype == SPARK_DTYPE_F16)
        k_silu_mul<__half><<<grid, 256, 0, s>>>((const __half*)gate, (const __half*)up, (__half*)out, n);
    else
        return set_error(SPARK_ERR_INVALID, "spark_silu_mul: bad dtype %d", dtype);
    return check_launch("spark_silu_mul");
}

int spark_silu_mul_rows(const void* gate, const void* up, int64_t ld_in, void* out, int64_t ld_out, int dtype,
                        int64_t rows, int64_t cols, void* stream) {
    SPARK_REQUIRE(gate && up && out && rows >= 0 && cols >= 0, SPARK_ERR_INVALID, "spark_silu_mul_rows: null pointer");
    SPARK_REQUIRE(ld_in >= cols && ld_out >= cols, SPARK_ERR_INVALID, "spark_silu_mul_rows: leading dimension below cols");
    const int64_t n = rows * cols;
    if (n == 0) return SPARK_OK;
    int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SPARK_DTYPE_F32)
        k_silu_mul_rows<float><<<grid, 256, 0, s>>>((const float*)gate, (const float*)up, ld_in, (float*)out, ld_out,
                                                    rows, cols);
    else if (dtype == SPARK_DTYPE_BF16)
        k_silu_mul_rows<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)gate, (const __nv_bfloat16*)up,
                                                            ld_in, (__nv_bfloat16*)out, ld_out, rows, cols);
    else if (dtype == SPARK_DTYPE_F16)
        k_silu_mul_rows<__half><<<grid, 256, 0, s>>>((const __half*)gate, (const __half*)up, ld_in, (__half*)out,
                                                     ld_out, rows, cols);
    else
        return set_error(SPARK_ERR_INVALID, "spark_silu_mul_rows: bad dtype %d", dtype);
    return check_launch("spark_silu_mul_rows");
}

}  // extern "C"
