// common.cuh -- shared device/host helpers for the SPARK B200 kernels.
//
// Everything here is written for sm_100a.  Format facts restated from the
// reference emulators (DJAzzs/SPARK 01_core/*.py) are cited where used.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/spark_b200.h"

namespace spark {

// ------------------------------------------------------------------ errors
// Host-side error recording (thread-local message, returned by
// spark_last_error()).
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

#define SPARK_REQUIRE(cond, code, ...)                      \
    do {                                                    \
        if (!(cond)) return ::spark::set_error((code), __VA_ARGS__); \
    } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------------ dtypes
__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
    if (dtype == SPARK_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
    if (dtype == SPARK_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_from_float(void* p, int dtype, int64_t i, float v) {
    if (dtype == SPARK_DTYPE_F32) reinterpret_cast<float*>(p)[i] = v;
    else if (dtype == SPARK_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

// ------------------------------------------------------------------ SPFP2
// Decoded SPFP2 magnitude 2^(e-10), e in [0,15] (block_fp2_emu.py:25).
__device__ __forceinline__ float spfp2_scale(int e) { return __uint_as_float((uint32_t)(117 + e) << 23); }

// Decision boundaries of the window centre c = round(log2(maxv) + 10 - 0.75)
// (block_fp2_emu.py:113-115) as evaluated by torch on the CPU: c is the
// number of thresholds <= the fp32 bit pattern of maxv.  The table was
// measured by bisection against torch.log2 (whose rounding differs from a
// correctly rounded log2 near these points).
__constant__ __device__ static const uint32_t kCenterThreshold[15] = {
    0x3b1837f4u, 0x3b9837efu, 0x3c1837f2u, 0x3c9837efu, 0x3d1837f2u,
    0x3d9837eeu, 0x3e1837f3u, 0x3e9837edu, 0x3f1837f4u, 0x3f9837edu,
    0x401837f5u, 0x409837edu, 0x411837f5u, 0x419837ecu, 0x421837f6u};

__device__ __forceinline__ int spfp2_center(float maxv) {
    // NaN / +inf -> 0 (the reference's .long() of a non-finite value is
    // INT64_MIN, clamped to 0).
    if (!(maxv <= 3.4028235e38f)) return 0;
    uint32_t b = __float_as_uint(maxv);
    int c = 0;
#pragma unroll
    for (int k = 0; k < 15; ++k) c += (b >= kCenterThreshold[k]);
    return c;
}

// ------------------------------------------------------------------ float8 e4m3fn
// Round-to-nearest-even float -> e4m3fn with subnormals; magnitudes above 464
// (and NaN / inf) become NaN (0x7f | sign), matching torch's non-saturating
// .to(torch.float8_e4m3fn) used by fp3_emu.py:119 and nvfp4_emu.py:96.  The
// hardware cvt.satfinite would clamp to 448 instead, so this is done with
// integer arithmetic.
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
    uint32_t u = __float_as_uint(x);
    uint32_t sign = (u >> 24) & 0x80u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x43f00000u) return (uint8_t)(sign | 0x7fu);       // >= 480, inf, NaN
    if (a < 0x3c800000u) {                                       // < 2^-6: subnormal grid 2^-9
        float v = __uint_as_float(a) * 512.0f;                   // exact
        uint32_t r = (uint32_t)__float2uint_rn(v);               // RNE, 0..8
        return (uint8_t)(sign | r);
    }
    uint32_t exp = (a >> 23) - 120u;                              // biased e4m3 exponent 1..15
    uint32_t mant = a & 0x7fffffu;
    uint32_t keep = mant >> 20;
    uint32_t rest = mant & 0xfffffu;
    if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) {
        keep += 1u;
        if (keep == 8u) { keep = 0u; exp += 1u; }
    }
    uint32_t code = (exp << 3) | keep;
    if (code >= 0x7fu) code = 0x7fu;
    return (uint8_t)(sign | code);
}

// e4m3fn -> float; NaN gets torch's bit pattern (0x7ff00000 | sign).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
    uint32_t sign = (b & 0x80u) << 24;
    uint32_t e = (b >> 3) & 0xfu, m = b & 7u;
    if (e == 0xfu && m == 7u) return __uint_as_float(sign | 0x7ff00000u);
    if (e == 0u) {
        float v = (float)m * (1.0f / 512.0f);
        return __uint_as_float(__float_as_uint(v) | sign);
    }
    return __uint_as_float(sign | ((e + 120u) << 23) | (m << 20));
}

// ------------------------------------------------------------------ bounded waits
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Kernel-side error word (in the caller's workspace): first error wins.
__device__ __forceinline__ void report_device_error(int* flag, int code) {
    if (flag) atomicCAS(flag, 0, code);
}

}  // namespace spark
