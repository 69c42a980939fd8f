// quant.cu -- quantize / pack / decode / STE fake-quant kernels for the four
// SPARK weight formats, with their C-ABI entry points.
//
// One thread owns one packing unit (an SPFP2 pair of 8-blocks, an FP3/NVFP4
// 16-block, a 2:4 pair of 16-blocks).  All arithmetic is explicit IEEE fp32
// (__fadd_rn/__fmul_rn/__fdiv_rn), so no FMA contraction changes a rounding
// the reference emulators do not make.  These kernels are HBM-bound byte
// work: loads are 16-byte vectors where the layout allows, packed bytes are
// gathered in shared memory and written back as whole words.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace spark {

__device__ __forceinline__ bool aligned_dev(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t units) { return (int)((units + kThreads - 1) / kThreads); }

// ---------------------------------------------------------------- loads
// n consecutive elements of w starting at element `base` as fp32 (any dtype),
// with zero fill past `limit`.
template <int N>
__device__ __forceinline__ void load_block(const void* w, int dtype, int64_t base, int64_t limit, float* v) {
    if (dtype == SPARK_DTYPE_F32 && base + N <= limit && ((base & 3) == 0) &&
        aligned_dev(reinterpret_cast<const float*>(w) + base)) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + base);
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            float4 q = __ldg(p + i);
            v[4 * i] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
        }
        return;
    }
    if (dtype != SPARK_DTYPE_F32 && N % 8 == 0 && base + N <= limit && ((base & 7) == 0) &&
        aligned_dev(reinterpret_cast<const uint16_t*>(w) + base)) {
        // 8 bf16 / fp16 values per 16-byte load
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) + base);
#pragma unroll
        for (int i = 0; i < N / 8; ++i) {
            const uint4 q = __ldg(p + i);
            const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (dtype == SPARK_DTYPE_BF16) {
                    v[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
                    v[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
                } else {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
                    v[8 * i + 2 * k] = f.x;
                    v[8 * i + 2 * k + 1] = f.y;
                }
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = (base + i < limit) ? load_as_float(w, dtype, base + i) : 0.0f;
}

// one row-padded 16-block: columns [16*cb, 16*cb+16) of row r, zero past ic
__device__ __forceinline__ void load_row_block16(const void* w, int dtype, int64_t r, int64_t cb, int64_t ic,
                                                 float* v) {
    int64_t c0 = cb * 16;
    if (c0 + 16 <= ic) {
        load_block<16>(w, dtype, r * ic + c0, r * ic + c0 + 16, v);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = (c0 + i < ic) ? load_as_float(w, dtype, r * ic + c0 + i) : 0.0f;
    }
}

}  // namespace

// ---------------------------------------------------------------- SPFP2 search
// amax of |w| with NaN propagation followed by clamp_min(lo)
template <int N>
__device__ __forceinline__ float amax_clamp(const float* w, float lo) {
    float m = 0.0f;
    bool nan = false;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        float a = fabsf(w[i]);
        nan |= (a != a);
        m = fmaxf(m, a);
    }
    if (nan) return __uint_as_float(0x7fc00000u);
    return m < lo ? lo : m;
}

// sum of squared errors of an 8-block at exponent e, sequential fp32
// (block_fp2_emu.py:118-124)
__device__ __forceinline__ float spfp2_err8(const float* w, int e) {
    const float s = spfp2_scale(e);
    const float half = __fmul_rn(s, 0.5f);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float q = fabsf(w[i]) > half ? (w[i] > 0.0f ? s : -s) : 0.0f;
        float d = __fsub_rn(w[i], q);
        acc = __fadd_rn(acc, __fmul_rn(d, d));
    }
    return acc;
}

// window search (block_fp2_emu.py:109-131) including the reference's start
// state: best = c, best_err = err(clamp(c-2)).
__device__ __forceinline__ int spfp2_search8(const float* w) {
    const int c = spfp2_center(amax_clamp<8>(w, 1e-38f));
    int best = c;
    float best_err = spfp2_err8(w, max(c - 2, 0));
#pragma unroll
    for (int off = -1; off <= 2; ++off) {
        int e = min(max(c + off, 0), 15);
        float err = spfp2_err8(w, e);
        if (err < best_err) { best = e; best_err = err; }
    }
    return best;
}

// mantissa word: code 0 (+1) if w > s/2, 1 (-1) if w < -s/2, else 2
// (block_fp2_emu.py:39-46)
__device__ __forceinline__ uint32_t spfp2_mword(const float* w, int e) {
    const float half = __fmul_rn(spfp2_scale(e), 0.5f);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t code = w[i] > half ? 0u : (w[i] < -half ? 1u : 2u);
        m |= code << (2 * i);
    }
    return m;
}

__device__ __forceinline__ void spfp2_decode8(uint32_t m, int e, float* out) {
    const float s = spfp2_scale(e);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t c = (m >> (2 * i)) & 3u;
        out[i] = c == 0 ? s : (c == 1 ? -s : 0.0f);
    }
}

// ---------------------------------------------------------------- SPFP2 kernels
// pack_blockwise_paired: thread = pair of blocks; 5 bytes per pair gathered in
// shared memory and stored as words.
__global__ void __launch_bounds__(kThreads) k_spfp2_pack_paired(const void* __restrict__ w, int dtype, int64_t n,
                                                                 uint8_t* __restrict__ packed,
                                                                 uint8_t* __restrict__ expv) {
    __shared__ __align__(16) uint8_t sbuf[kThreads * 5];
    const int64_t nb = n / 8;
    const int64_t np = (nb + 1) / 2;
    const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (p < np) {
        uint32_t m[2] = {0u, 0u};
        int e[2] = {0, 0};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int64_t b = 2 * p + h;
            if (b < nb) {
                float v[8];
                load_block<8>(w, dtype, b * 8, n, v);
                e[h] = spfp2_search8(v);
                m[h] = spfp2_mword(v, e[h]);
                if (expv) expv[b] = (uint8_t)e[h];
            }
        }
        uint8_t* o = sbuf + threadIdx.x * 5;
        o[0] = (uint8_t)(m[0] & 0xff);
        o[1] = (uint8_t)(m[0] >> 8);
        o[2] = (uint8_t)(m[1] & 0xff);
        o[3] = (uint8_t)(m[1] >> 8);
        o[4] = (uint8_t)(e[0] | (e[1] << 4));
    }
    __syncthreads();
    const int64_t p0 = (int64_t)blockIdx.x * kThreads;
    const int64_t nbytes = min((int64_t)kThreads, np - p0) * 5;
    uint8_t* dst = packed + p0 * 5;
    if (nbytes == kThreads * 5 && aligned_dev(dst)) {
        const uint4* s4 = reinterpret_cast<const uint4*>(sbuf);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (int i = threadIdx.x; i < kThreads * 5 / 16; i += kThreads) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < nbytes; i += kThreads) dst[i] = sbuf[i];
    }
}

// pack_blockwise_search (3-byte v1): thread = one block
__global__ void __launch_bounds__(kThreads) k_spfp2_pack_v1(const void* __restrict__ w, int dtype, int64_t n,
                                                             uint8_t* __restrict__ packed,
                                                             uint8_t* __restrict__ expv) {
    const int64_t nb = n / 8;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= nb) return;
    float v[8];
    load_block<8>(w, dtype, b * 8, n, v);
    int e = spfp2_search8(v);
    uint32_t m = spfp2_mword(v, e);
    packed[3 * b] = (uint8_t)(m & 0xff);
    packed[3 * b + 1] = (uint8_t)(m >> 8);
    packed[3 * b + 2] = (uint8_t)e;
    if (expv) expv[b] = (uint8_t)e;
}

__global__ void __launch_bounds__(kThreads) k_spfp2_unpack_paired(const uint8_t* __restrict__ packed,
                                                                   int64_t n_pairs, int64_t n_elements,
                                                                   void* __restrict__ out, int dtype) {
    const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (p >= n_pairs) return;
    const uint8_t* q = packed + 5 * p;
    float v[16];
    spfp2_decode8((uint32_t)q[0] | ((uint32_t)q[1] << 8), q[4] & 0xf, v);
    spfp2_decode8((uint32_t)q[2] | ((uint32_t)q[3] << 8), q[4] >> 4, v + 8);
    const int64_t base = p * 16;
    if (dtype == SPARK_DTYPE_F32 && base + 16 <= n_elements && aligned_dev(reinterpret_cast<float*>(out) + base)) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + base);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (base + i < n_elements) store_from_float(out, dtype, base + i, v[i]);
}

__global__ void __launch_bounds__(kThreads) k_spfp2_unpack_v1(const uint8_t* __restrict__ packed, int64_t nb,
                                                               void* __restrict__ out, int dtype) {
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= nb) return;
    float v[8];
    spfp2_decode8((uint32_t)packed[3 * b] | ((uint32_t)packed[3 * b + 1] << 8), packed[3 * b + 2] & 0xf, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) store_from_float(out, dtype, b * 8 + i, v[i]);
}

// Legacy single-exponent blocks read by the reference's decode_fp32 /
// decode_fp16 ops (01_core/block_fp2_kernel.cu:3-34): 5 bytes per 16 weights,
// bytes 0-3 a little-endian word of 16 2-bit codes (code j at bits 2j), byte 4
// the exponent in its low nibble (the high nibble is ignored); value =
// (+1, -1, 0, 0)[code] * 2^(e-10).
__global__ void __launch_bounds__(kThreads) k_spfp2_legacy_decode(const uint8_t* __restrict__ packed, int64_t nb,
                                                                   void* __restrict__ out, int dtype) {
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= nb) return;
    const uint8_t* q = packed + 5 * b;
    float v[16];
    spfp2_decode8((uint32_t)q[0] | ((uint32_t)q[1] << 8), q[4] & 0xf, v);
    spfp2_decode8((uint32_t)q[2] | ((uint32_t)q[3] << 8), q[4] & 0xf, v + 8);
#pragma unroll
    for (int i = 0; i < 16; ++i) store_from_float(out, dtype, b * 16 + i, v[i]);
}

// channel_fake_quantize forward: search + 3-byte decode per flattened 8-block
// (block_fp2_emu.py:365-375).  With `twofour`, two_four_apply follows on each
// group of 4 (two_four.py:70-75): the first two nonzeros survive and dropped
// values are multiplied by 0.0 (a dropped negative becomes -0.0).
__global__ void __launch_bounds__(kThreads) k_spfp2_fake_quant(const void* __restrict__ w, int in_dtype, int64_t n,
                                                                void* __restrict__ out, int out_dtype, int twofour) {
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= n / 8) return;
    float v[8], d[8];
    load_block<8>(w, in_dtype, b * 8, n, v);
    int e = spfp2_search8(v);
    spfp2_decode8(spfp2_mword(v, e), e, d);
    if (twofour) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            int kept = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float& x = d[4 * g + i];
                if (x != 0.0f) {
                    if (kept < 2) ++kept;
                    else x = __fmul_rn(x, 0.0f);
                }
            }
        }
    }
    const int64_t base = b * 8;
    if (out_dtype == SPARK_DTYPE_F32 && aligned_dev(reinterpret_cast<float*>(out) + base)) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + base);
        o[0] = make_float4(d[0], d[1], d[2], d[3]);
        o[1] = make_float4(d[4], d[5], d[6], d[7]);
        return;
    }
    if (out_dtype != SPARK_DTYPE_F32 && aligned_dev(reinterpret_cast<uint16_t*>(out) + base)) {
        uint32_t u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (out_dtype == SPARK_DTYPE_BF16) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(d[2 * k], d[2 * k + 1]);
                u[k] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
                const __half2 h = __floats2half2_rn(d[2 * k], d[2 * k + 1]);
                u[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + base) = make_uint4(u[0], u[1], u[2], u[3]);
        return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) store_from_float(out, out_dtype, base + i, d[i]);
}

// ---------------------------------------------------------------- FP3 / NVFP4
// bucketize(|x|, bounds, right=False) = number of bounds strictly below |x|;
// NaN goes to the last bucket (fp3_emu.py:122, nvfp4_emu.py:99).
__device__ __forceinline__ int fp3_mag(float ax) {
    if (ax != ax) return 3;
    return (ax > 0.25f) + (ax > 0.75f) + (ax > 1.25f);
}
__device__ __forceinline__ int e2m1_idx(float ax) {
    if (ax != ax) return 7;
    return (ax > 0.25f) + (ax > 0.75f) + (ax > 1.25f) + (ax > 1.75f) + (ax > 2.5f) + (ax > 3.5f) + (ax > 5.0f);
}

// block scale: fp8(clamp_min(amax / top, 1e-30)) (fp3_emu.py:117-119, nvfp4_emu.py:94-96)
__device__ __forceinline__ uint8_t block_scale(const float* v, float top, float* s) {
    float amax = amax_clamp<16>(v, 0.0f);
    float sf = __fdiv_rn(amax, top);
    if (!(sf >= 1e-30f) && !(sf != sf)) sf = 1e-30f;
    uint8_t s8 = f32_to_e4m3(sf);
    *s = e4m3_to_f32(s8);
    return s8;
}

__constant__ float kFp3Table[8] = {0.0f, 0.5f, 1.0f, 1.5f, -0.0f, -0.5f, -1.0f, -1.5f};  // fp3_emu.py:47
__constant__ float kE2m1Pos[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};      // nvfp4_emu.py:20

// code value times block scale.  A NaN scale propagates its own bits, as the
// x86 multiply behind the reference does (the GPU would return a canonical NaN).
__device__ __forceinline__ float scaled(float v, float s) { return (s != s) ? s : __fmul_rn(v, s); }

// FP3 codes of one 16-block (sign<<2 | mag)
__device__ __forceinline__ void fp3_codes16(const float* v, float s, uint32_t* c) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float xs = __fdiv_rn(v[i], s);
        c[i] = ((xs < 0.0f) ? 4u : 0u) | (uint32_t)fp3_mag(fabsf(xs));
    }
}

// thread = one row-padded 16-block.  layout 0: 3-bit groups (6 B / block),
// layout 1: nibbles (8 B / block).
__global__ void __launch_bounds__(kThreads) k_fp3_pack(const void* __restrict__ w, int dtype, int64_t oc, int64_t ic,
                                                       uint8_t* __restrict__ codes, uint8_t* __restrict__ scales,
                                                       int nibble) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    float v[16];
    load_row_block16(w, dtype, b / nbr, b % nbr, ic, v);
    float s;
    scales[b] = block_scale(v, 1.5f, &s);
    uint32_t c[16];
    fp3_codes16(v, s, c);
    if (nibble) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) lo |= (c[i] & 0xf) << (4 * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) hi |= (c[8 + i] & 0xf) << (4 * i);
        uint8_t* o = codes + 8 * b;
        if (((uintptr_t)o & 7) == 0) {
            *reinterpret_cast<uint2*>(o) = make_uint2(lo, hi);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) { o[k] = (uint8_t)(lo >> (8 * k)); o[4 + k] = (uint8_t)(hi >> (8 * k)); }
        }
    } else {
        uint32_t g0 = 0, g1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) { g0 |= c[i] << (3 * i); g1 |= c[8 + i] << (3 * i); }
        uint8_t* o = codes + 6 * b;
        o[0] = (uint8_t)g0; o[1] = (uint8_t)(g0 >> 8); o[2] = (uint8_t)(g0 >> 16);
        o[3] = (uint8_t)g1; o[4] = (uint8_t)(g1 >> 8); o[5] = (uint8_t)(g1 >> 16);
    }
}

__global__ void __launch_bounds__(kThreads) k_fp3_unpack(const uint8_t* __restrict__ codes,
                                                         const uint8_t* __restrict__ scales, int64_t oc, int64_t ic,
                                                         void* __restrict__ out, int dtype, int nibble) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    const float s = e4m3_to_f32(scales[b]);
    uint32_t c[16];
    if (nibble) {
        const uint8_t* q = codes + 8 * b;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            uint32_t nib = (i & 1) ? (q[i / 2] >> 4) : (q[i / 2] & 0xf);
            c[i] = nib > 7 ? 7 : nib;                                  // fp3_emu.py:84 clamp(max=7)
        }
    } else {
        const uint8_t* q = codes + 6 * b;
        uint32_t g0 = q[0] | (q[1] << 8) | (q[2] << 16), g1 = q[3] | (q[4] << 8) | (q[5] << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) { c[i] = (g0 >> (3 * i)) & 7; c[8 + i] = (g1 >> (3 * i)) & 7; }
    }
    const int64_t r = b / nbr, c0 = (b % nbr) * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (c0 + i < ic) store_from_float(out, dtype, r * ic + c0 + i, scaled(kFp3Table[c[i]], s));
}

__global__ void __launch_bounds__(kThreads) k_fp3_fake_quant(const void* __restrict__ w, int in_dtype, int64_t oc,
                                                             int64_t ic, void* __restrict__ out, int out_dtype) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    float v[16];
    const int64_t r = b / nbr, c0 = (b % nbr) * 16;
    load_row_block16(w, in_dtype, r, b % nbr, ic, v);
    float s;
    block_scale(v, 1.5f, &s);
    uint32_t c[16];
    fp3_codes16(v, s, c);
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (c0 + i < ic) store_from_float(out, out_dtype, r * ic + c0 + i, scaled(kFp3Table[c[i]], s));
}

__global__ void __launch_bounds__(kThreads) k_nvfp4_pack(const void* __restrict__ w, int dtype, int64_t oc,
                                                         int64_t ic, uint8_t* __restrict__ codes,
                                                         uint8_t* __restrict__ scales) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    float v[16];
    load_row_block16(w, dtype, b / nbr, b % nbr, ic, v);
    float s;
    scales[b] = block_scale(v, 6.0f, &s);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float xs = __fdiv_rn(v[i], s);
        uint32_t code = (uint32_t)e2m1_idx(fabsf(xs)) + (xs < 0.0f ? 8u : 0u);
        if (i < 8) lo |= code << (4 * i);
        else hi |= code << (4 * (i - 8));
    }
    uint8_t* o = codes + 8 * b;
    if (((uintptr_t)o & 7) == 0) {
        *reinterpret_cast<uint2*>(o) = make_uint2(lo, hi);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) { o[k] = (uint8_t)(lo >> (8 * k)); o[4 + k] = (uint8_t)(hi >> (8 * k)); }
    }
}

__global__ void __launch_bounds__(kThreads) k_nvfp4_unpack(const uint8_t* __restrict__ codes,
                                                           const uint8_t* __restrict__ scales, int64_t oc,
                                                           int64_t ic, void* __restrict__ out, int dtype) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    const float s = e4m3_to_f32(scales[b]);
    const uint8_t* q = codes + 8 * b;
    const int64_t r = b / nbr, c0 = (b % nbr) * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        uint32_t code = (i & 1) ? (q[i / 2] >> 4) : (q[i / 2] & 0xf);
        float v = code < 8 ? kE2m1Pos[code] : -kE2m1Pos[code - 8];
        if (c0 + i < ic) store_from_float(out, dtype, r * ic + c0 + i, scaled(v, s));
    }
}

// NVFP4 embedding lookup: out[i, :] = decode(row ids[i]) of a packed
// [num_embeddings, dim] table -- the forward of NVFP4EmbeddingQAT
// (quant_linear.py:507-537, F.embedding of the quantised table) reading only
// the looked-up rows' codes.  One thread per (id, 16-block), the arithmetic
// of k_nvfp4_unpack.  An id outside [0, num_embeddings) yields a zero row
// and records error code 7 in *err (the caller's workspace word).
__global__ void __launch_bounds__(kThreads) k_nvfp4_embedding(const uint8_t* __restrict__ codes,
                                                              const uint8_t* __restrict__ scales, int64_t rows,
                                                              int64_t dim, const int64_t* __restrict__ ids,
                                                              int64_t n_ids, void* __restrict__ out, int dtype,
                                                              int* err) {
    const int64_t nbr = (dim + 15) / 16;
    const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (t >= n_ids * nbr) return;
    const int64_t i = t / nbr, blk = t - i * nbr, c0 = blk * 16;
    const int64_t r = ids[i];
    if (r < 0 || r >= rows) {
        if (blk == 0) report_device_error(err, 7);
        for (int k = 0; k < 16; ++k)
            if (c0 + k < dim) store_from_float(out, dtype, i * dim + c0 + k, 0.0f);
        return;
    }
    const int64_t b = r * nbr + blk;
    const float s = e4m3_to_f32(scales[b]);
    const uint8_t* q = codes + 8 * b;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const uint32_t code = (k & 1) ? (q[k / 2] >> 4) : (q[k / 2] & 0xf);
        const float v = code < 8 ? kE2m1Pos[code] : -kE2m1Pos[code - 8];
        if (c0 + k < dim) store_from_float(out, dtype, i * dim + c0 + k, scaled(v, s));
    }
}

// nvfp4_fake_quant: sign(x) * E2M1(|x|) * s with sign(NaN) = 0 (nvfp4_emu.py:26-30)
__global__ void __launch_bounds__(kThreads) k_nvfp4_fake_quant(const void* __restrict__ w, int in_dtype, int64_t oc,
                                                               int64_t ic, void* __restrict__ out, int out_dtype) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t b = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (b >= oc * nbr) return;
    float v[16];
    const int64_t r = b / nbr, c0 = (b % nbr) * 16;
    load_row_block16(w, in_dtype, r, b % nbr, ic, v);
    float s;
    block_scale(v, 6.0f, &s);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float xs = __fdiv_rn(v[i], s);
        float q = kE2m1Pos[e2m1_idx(fabsf(xs))];
        float sg = xs > 0.0f ? 1.0f : (xs < 0.0f ? -1.0f : 0.0f);
        if (c0 + i < ic) store_from_float(out, out_dtype, r * ic + c0 + i, scaled(__fmul_rn(sg, q), s));
    }
}

// ---------------------------------------------------------------- 2:4
// 16-block error at exponent e: lanes k and k+8 summed first, then the 8 lane
// sums sequentially (the order of torch's full .sum(), two_four.py:106)
__device__ __forceinline__ float tf_err16(const float* w, int e) {
    const float s = spfp2_scale(e);
    const float half = __fmul_rn(s, 0.5f);
    float d2[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float q = fabsf(w[i]) > half ? (w[i] > 0.0f ? s : -s) : 0.0f;
        float d = __fsub_rn(w[i], q);
        d2[i] = __fmul_rn(d, d);
    }
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = __fadd_rn(acc, __fadd_rn(d2[k], d2[k + 8]));
    return acc;
}

// _search_exp (two_four.py:98-109): the first candidate is always taken
__device__ __forceinline__ int tf_search16(const float* w) {
    const int c = spfp2_center(amax_clamp<16>(w, 1e-38f));
    int best = max(c - 2, 0);
    float best_err = tf_err16(w, best);
#pragma unroll
    for (int off = -1; off <= 2; ++off) {
        int e = min(max(c + off, 0), 15);
        float err = tf_err16(w, e);
        if (err < best_err) { best = e; best_err = err; }
    }
    return best;
}

// mode index of the pair (a, b), a < b: (0,1)(0,2)(0,3)(1,2)(1,3)(2,3) (two_four.py:23)
__device__ __forceinline__ uint32_t tf_dual(int a, int b) { return a == 0 ? (uint32_t)(b - 1) : (a == 1 ? (uint32_t)(b + 1) : 5u); }

// 28-bit slot code of one 16-block (two_four.py:136-147)
__device__ __forceinline__ uint32_t tf_encode16(const float* w, int e) {
    const float half = __fmul_rn(spfp2_scale(e), 0.5f);
    uint32_t v = (uint32_t)e << 24;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        int cnt = 0, p0 = 0, p1 = 0;
        uint32_t n0 = 0, n1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float x = w[4 * g + i];
            if (fabsf(x) > half) {
                uint32_t neg = x < 0.0f;
                if (cnt == 0) { p0 = i; n0 = neg; }
                else if (cnt == 1) { p1 = i; n1 = neg; }
                ++cnt;
            }
        }
        uint32_t mode = cnt == 0 ? 15u : (cnt == 1 ? 8u + (uint32_t)p0 : tf_dual(p0, p1));
        if (cnt == 1) n1 = 0;
        if (cnt == 0) { n0 = 0; n1 = 0; }
        v |= mode << (4 * g);
        v |= n0 << (16 + 2 * g);
        v |= n1 << (17 + 2 * g);
    }
    return v;
}

// thread = pair of 16-blocks (7 bytes)
__global__ void __launch_bounds__(kThreads) k_twofour_pack(const void* __restrict__ w, int dtype, int64_t oc,
                                                           int64_t ic, uint8_t* __restrict__ packed) {
    const int64_t nbr = (ic + 15) / 16;
    const int64_t nb = oc * nbr;
    const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (p >= (nb + 1) / 2) return;
    uint64_t v = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int64_t b = 2 * p + h;
        float blk[16];
        if (b < nb) load_row_block16(w, dtype, b / nbr, b % nbr, ic, blk);
        else {
#pragma unroll
            for (int i = 0; i < 16; ++i) blk[i] = 0.0f;
        }
        int e = tf_search16(blk);
        v |= (uint64_t)tf_encode16(blk, e) << (28 * h);
    }
    uint8_t* o = packed + 7 * p;
#pragma unroll
    for (int k = 0; k < 7; ++k) o[k] = (uint8_t)(v >> (8 * k));
}

__global__ void __launch_bounds__(kThreads) k_twofour_unpack(const uint8_t* __restrict__ packed, int64_t n_pairs,
                                                             int64_t n_elements, void* __restrict__ out, int dtype) {
    const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (p >= n_pairs) return;
    uint64_t v = 0;
#pragma unroll
    for (int k = 0; k < 7; ++k) v |= (uint64_t)packed[7 * p + k] << (8 * k);
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
        uint32_t word = (uint32_t)(v >> (28 * slot)) & 0x0fffffffu;
        const float s = spfp2_scale((word >> 24) & 0xf);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint32_t mode = (word >> (4 * g)) & 0xf;
            float n0 = ((word >> (16 + 2 * g)) & 1) ? -s : s;
            float n1 = ((word >> (17 + 2 * g)) & 1) ? -s : s;
            float vals[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (mode < 6) {
                int a = mode < 3 ? 0 : (mode < 5 ? 1 : 2);
                int b = mode == 0 ? 1 : (mode == 1 ? 2 : (mode == 2 ? 3 : (mode == 3 ? 2 : 3)));
                vals[a] = n0;
                vals[b] = n1;
            } else if (mode >= 8 && mode <= 11) {
                vals[mode - 8] = n0;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                int64_t idx = p * 32 + slot * 16 + g * 4 + i;
                if (idx < n_elements) store_from_float(out, dtype, idx, vals[i]);
            }
        }
    }
}

}  // namespace spark

// ====================================================================== C ABI
using namespace spark;

namespace {
inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool dtype_ok(int d) { return d == SPARK_DTYPE_F32 || d == SPARK_DTYPE_BF16 || d == SPARK_DTYPE_F16; }
}  // namespace

extern "C" {

int spark_spfp2_pack(const void* w, int w_dtype, int64_t n, uint8_t* packed, uint8_t* expv, void* stream) {
    SPARK_REQUIRE(w && packed && n >= 0, SPARK_ERR_INVALID, "spark_spfp2_pack: null pointer or negative size");
    SPARK_REQUIRE(n % 8 == 0, SPARK_ERR_INVALID, "spark_spfp2_pack: numel %lld is not a multiple of 8", (long long)n);
    SPARK_REQUIRE(dtype_ok(w_dtype), SPARK_ERR_INVALID, "spark_spfp2_pack: bad dtype %d", w_dtype);
    int64_t np = (n / 8 + 1) / 2;
    if (np == 0) return SPARK_OK;
    k_spfp2_pack_paired<<<grid_for(np), kThreads, 0, S(stream)>>>(w, w_dtype, n, packed, expv);
    return check_launch("spark_spfp2_pack");
}

int spark_spfp2_pack_v1(const void* w, int w_dtype, int64_t n, uint8_t* packed, uint8_t* expv, void* stream) {
    SPARK_REQUIRE(w && packed && n >= 0, SPARK_ERR_INVALID, "spark_spfp2_pack_v1: null pointer or negative size");
    SPARK_REQUIRE(n % 8 == 0, SPARK_ERR_INVALID, "spark_spfp2_pack_v1: numel %lld is not a multiple of 8", (long long)n);
    SPARK_REQUIRE(dtype_ok(w_dtype), SPARK_ERR_INVALID, "spark_spfp2_pack_v1: bad dtype %d", w_dtype);
    if (n == 0) return SPARK_OK;
    k_spfp2_pack_v1<<<grid_for(n / 8), kThreads, 0, S(stream)>>>(w, w_dtype, n, packed, expv);
    return check_launch("spark_spfp2_pack_v1");
}

int spark_spfp2_unpack(const uint8_t* packed, int64_t n_elements, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(packed && out && n_elements >= 0, SPARK_ERR_INVALID, "spark_spfp2_unpack: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_spfp2_unpack: bad dtype %d", out_dtype);
    int64_t np = (n_elements + 15) / 16;
    if (np == 0) return SPARK_OK;
    k_spfp2_unpack_paired<<<grid_for(np), kThreads, 0, S(stream)>>>(packed, np, n_elements, out, out_dtype);
    return check_launch("spark_spfp2_unpack");
}

int spark_spfp2_unpack_v1(const uint8_t* packed, int64_t n_blocks, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(packed && out && n_blocks >= 0, SPARK_ERR_INVALID, "spark_spfp2_unpack_v1: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_spfp2_unpack_v1: bad dtype %d", out_dtype);
    if (n_blocks == 0) return SPARK_OK;
    k_spfp2_unpack_v1<<<grid_for(n_blocks), kThreads, 0, S(stream)>>>(packed, n_blocks, out, out_dtype);
    return check_launch("spark_spfp2_unpack_v1");
}

int spark_spfp2_legacy_decode(const uint8_t* packed, int64_t n_blocks, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(packed && out && n_blocks >= 0, SPARK_ERR_INVALID, "spark_spfp2_legacy_decode: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_spfp2_legacy_decode: bad dtype %d", out_dtype);
    if (n_blocks == 0) return SPARK_OK;
    k_spfp2_legacy_decode<<<grid_for(n_blocks), kThreads, 0, S(stream)>>>(packed, n_blocks, out, out_dtype);
    return check_launch("spark_spfp2_legacy_decode");
}

int spark_spfp2_fake_quant(const void* w, int w_dtype, int64_t n, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(w && out && n >= 0, SPARK_ERR_INVALID, "spark_spfp2_fake_quant: null pointer");
    SPARK_REQUIRE(n % 8 == 0, SPARK_ERR_INVALID, "spark_spfp2_fake_quant: numel %lld is not a multiple of 8", (long long)n);
    SPARK_REQUIRE(dtype_ok(w_dtype) && dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_spfp2_fake_quant: bad dtype");
    if (n == 0) return SPARK_OK;
    k_spfp2_fake_quant<<<grid_for(n / 8), kThreads, 0, S(stream)>>>(w, w_dtype, n, out, out_dtype, 0);
    return check_launch("spark_spfp2_fake_quant");
}

static int fp3_pack_impl(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                         void* stream, int nibble, const char* name) {
    SPARK_REQUIRE(w && codes && scales && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "%s: null pointer or negative size", name);
    SPARK_REQUIRE(dtype_ok(w_dtype), SPARK_ERR_INVALID, "%s: bad dtype %d", name, w_dtype);
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_fp3_pack<<<grid_for(nb), kThreads, 0, S(stream)>>>(w, w_dtype, oc, ic, codes, scales, nibble);
    return check_launch(name);
}

int spark_fp3_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales, void* stream) {
    return fp3_pack_impl(w, w_dtype, oc, ic, codes, scales, stream, 0, "spark_fp3_pack");
}

int spark_fp3_pack_nibble(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                          void* stream) {
    return fp3_pack_impl(w, w_dtype, oc, ic, codes, scales, stream, 1, "spark_fp3_pack_nibble");
}

static int fp3_unpack_impl(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                           int out_dtype, void* stream, int nibble, const char* name) {
    SPARK_REQUIRE(codes && scales && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "%s: null pointer", name);
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "%s: bad dtype %d", name, out_dtype);
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_fp3_unpack<<<grid_for(nb), kThreads, 0, S(stream)>>>(codes, scales, oc, ic, out, out_dtype, nibble);
    return check_launch(name);
}

int spark_fp3_unpack(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out, int out_dtype,
                     void* stream) {
    return fp3_unpack_impl(codes, scales, oc, ic, out, out_dtype, stream, 0, "spark_fp3_unpack");
}

int spark_fp3_unpack_nibble(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                            int out_dtype, void* stream) {
    return fp3_unpack_impl(codes, scales, oc, ic, out, out_dtype, stream, 1, "spark_fp3_unpack_nibble");
}

int spark_fp3_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(w && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_fp3_fake_quant: null pointer");
    SPARK_REQUIRE(dtype_ok(w_dtype) && dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_fp3_fake_quant: bad dtype");
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_fp3_fake_quant<<<grid_for(nb), kThreads, 0, S(stream)>>>(w, w_dtype, oc, ic, out, out_dtype);
    return check_launch("spark_fp3_fake_quant");
}

int spark_nvfp4_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales,
                     void* stream) {
    SPARK_REQUIRE(w && codes && scales && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_nvfp4_pack: null pointer");
    SPARK_REQUIRE(dtype_ok(w_dtype), SPARK_ERR_INVALID, "spark_nvfp4_pack: bad dtype %d", w_dtype);
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_nvfp4_pack<<<grid_for(nb), kThreads, 0, S(stream)>>>(w, w_dtype, oc, ic, codes, scales);
    return check_launch("spark_nvfp4_pack");
}

int spark_nvfp4_unpack(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, void* out,
                       int out_dtype, void* stream) {
    SPARK_REQUIRE(codes && scales && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_nvfp4_unpack: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_nvfp4_unpack: bad dtype %d", out_dtype);
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_nvfp4_unpack<<<grid_for(nb), kThreads, 0, S(stream)>>>(codes, scales, oc, ic, out, out_dtype);
    return check_launch("spark_nvfp4_unpack");
}

int spark_nvfp4_embedding(const uint8_t* codes, const uint8_t* scales, int64_t num_embeddings, int64_t dim,
                          const int64_t* ids, int64_t n_ids, void* out, int out_dtype, int* err, void* stream) {
    SPARK_REQUIRE(num_embeddings >= 0 && dim >= 0 && n_ids >= 0, SPARK_ERR_INVALID,
                  "spark_nvfp4_embedding: negative size");
    if (n_ids == 0 || dim == 0) return SPARK_OK;
    SPARK_REQUIRE(codes && scales && out && ids, SPARK_ERR_INVALID, "spark_nvfp4_embedding: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_nvfp4_embedding: bad dtype %d", out_dtype);
    const int64_t n = n_ids * ((dim + 15) / 16);
    if (n == 0) return SPARK_OK;
    k_nvfp4_embedding<<<grid_for(n), kThreads, 0, S(stream)>>>(codes, scales, num_embeddings, dim, ids, n_ids, out,
                                                               out_dtype, err);
    return check_launch("spark_nvfp4_embedding");
}

int spark_nvfp4_fake_quant(const void* w, int w_dtype, int64_t oc, int64_t ic, void* out, int out_dtype,
                           void* stream) {
    SPARK_REQUIRE(w && out && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_nvfp4_fake_quant: null pointer");
    SPARK_REQUIRE(dtype_ok(w_dtype) && dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_nvfp4_fake_quant: bad dtype");
    int64_t nb = oc * ((ic + 15) / 16);
    if (nb == 0) return SPARK_OK;
    k_nvfp4_fake_quant<<<grid_for(nb), kThreads, 0, S(stream)>>>(w, w_dtype, oc, ic, out, out_dtype);
    return check_launch("spark_nvfp4_fake_quant");
}

int spark_twofour_pack(const void* w, int w_dtype, int64_t oc, int64_t ic, uint8_t* packed, void* stream) {
    SPARK_REQUIRE(w && packed && oc >= 0 && ic >= 0, SPARK_ERR_INVALID, "spark_twofour_pack: null pointer");
    SPARK_REQUIRE(dtype_ok(w_dtype), SPARK_ERR_INVALID, "spark_twofour_pack: bad dtype %d", w_dtype);
    int64_t nb = oc * ((ic + 15) / 16);
    int64_t np = (nb + 1) / 2;
    if (np == 0) return SPARK_OK;
    k_twofour_pack<<<grid_for(np), kThreads, 0, S(stream)>>>(w, w_dtype, oc, ic, packed);
    return check_launch("spark_twofour_pack");
}

int spark_twofour_unpack(const uint8_t* packed, int64_t n_elements, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(packed && out && n_elements >= 0, SPARK_ERR_INVALID, "spark_twofour_unpack: null pointer");
    SPARK_REQUIRE(dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_twofour_unpack: bad dtype %d", out_dtype);
    int64_t np = (n_elements + 31) / 32;
    if (np == 0) return SPARK_OK;
    k_twofour_unpack<<<grid_for(np), kThreads, 0, S(stream)>>>(packed, np, n_elements, out, out_dtype);
    return check_launch("spark_twofour_unpack");
}

int spark_twofour_fake_quant(const void* w, int w_dtype, int64_t n, void* out, int out_dtype, void* stream) {
    SPARK_REQUIRE(w && out && n >= 0, SPARK_ERR_INVALID, "spark_twofour_fake_quant: null pointer");
    SPARK_REQUIRE(n % 8 == 0, SPARK_ERR_INVALID, "spark_twofour_fake_quant: numel %lld is not a multiple of 8", (long long)n);
    SPARK_REQUIRE(dtype_ok(w_dtype) && dtype_ok(out_dtype), SPARK_ERR_INVALID, "spark_twofour_fake_quant: bad dtype");
    if (n == 0) return SPARK_OK;
    k_spfp2_fake_quant<<<grid_for(n / 8), kThreads, 0, S(stream)>>>(w, w_dtype, n, out, out_dtype, 1);
    return check_launch("spark_twofour_fake_quant");
}

}  // extern "C"
