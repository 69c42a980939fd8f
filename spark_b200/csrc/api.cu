// api.cu -- error reporting and small utilities of the C ABI.
#include <stdarg.h>
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

}  // extern "C"
