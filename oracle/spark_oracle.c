/*
 * spark_oracle.c -- CPU restatement of SPARK's format emulators.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in spark_b200/.  Only tests/, __graft_entry__.smoke() and the CPU
 * baseline leg of bench.py may load it; the product path never does.
 *
 * Every function restates one reference function (path:line in the
 * DJAzzs/SPARK tree) in plain C so that the GPU kernels can be checked bit for
 * bit on inputs far larger than the torch emulators finish in seconds.  The
 * arithmetic mirrors what torch 2.11 (CPU, AVX512 dispatch) does for those
 * emulators:
 *   - fp32 everywhere, no FMA contraction (built with -ffp-contract=off);
 *   - 8-element row sums (block_fp2_emu.py:124) are sequential from 0;
 *   - the 16-element full sum in two_four.py:106 adds lane k and k+8 first,
 *     then accumulates the 8 lane sums sequentially from 0;
 *   - torch.log2 rounding is captured as exact fp32 bit thresholds for the
 *     window centre (see spo_spfp2_center);
 *   - float -> float8_e4m3fn is round-to-nearest-even with subnormals and
 *     magnitudes above 464 becoming NaN (never saturating);
 *   - torch.bucketize(right=False) counts boundaries strictly below |x|
 *     (ties go down) and sends NaN to the last bucket.
 * These facts were measured against the emulators in this repository's
 * tests/golden/make_golden.py run and are pinned by tests/test_oracle_golden.py.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define SPO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* bit helpers                                                               */
/* ------------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* 2^(e-10) for e in [0,15] -- block_fp2_emu.py:25 (BIAS = 10) */
static inline float spfp2_scale(int e) { return u2f((uint32_t)(117 + e) << 23); }

/* ------------------------------------------------------------------------ */
/* SPFP2 window centre -- block_fp2_emu.py:113-115                           */
/*   c = round_half_even(fl(fl(log2(maxv)) + 10) - 0.75), clamped to [0,15]   */
/* torch's log2 is not correctly rounded; the exact decision boundaries      */
/* (smallest fp32 maxv with c >= k) were measured by bisection against       */
/* torch.log2 on the CPU and are identical at every tensor position.         */
/* NaN and +inf give 0 (torch casts them to INT64_MIN before the clamp).     */
/* ------------------------------------------------------------------------ */
static const uint32_t SPO_CENTER_T[15] = {
    0x3b1837f4u, 0x3b9837efu, 0x3c1837f2u, 0x3c9837efu, 0x3d1837f2u,
    0x3d9837eeu, 0x3e1837f3u, 0x3e9837edu, 0x3f1837f4u, 0x3f9837edu,
    0x401837f5u, 0x409837edu, 0x411837f5u, 0x419837ecu, 0x421837f6u};

SPO_API const uint32_t* spo_center_thresholds(void) { return SPO_CENTER_T; }

SPO_API int spo_spfp2_center(float maxv) {
    /* maxv is already clamp_min(1e-38)'d and non-negative (or NaN) */
    if (isnan(maxv) || isinf(maxv)) return 0;
    uint32_t b = f2u(maxv);
    int c = 0;
    for (int k = 0; k < 15; ++k) c += (b >= SPO_CENTER_T[k]);
    return c;
}

/* amax(|w|) with NaN propagation, then clamp_min(lo) (NaN stays NaN) */
static inline float amax_clamp(const float* w, int n, float lo) {
    float m = 0.0f;
    int nan = 0;
    for (int i = 0; i < n; ++i) {
        float a = fabsf(w[i]);
        if (isnan(a)) nan = 1;
        else if (a > m) m = a;
    }
    if (nan) return u2f(0x7fc00000u);
    return m < lo ? lo : m;
}

/* squared error of one 8-block against exponent e, sequential fp32 sum
 * -- block_fp2_emu.py:118-124 */
static float spfp2_err8(const float* w, int e) {
    const float s = spfp2_scale(e);
    const float half = s * 0.5f;
    float acc = 0.0f;
    for (int i = 0; i < 8; ++i) {
        float q = 0.0f;
        if (fabsf(w[i]) > half) q = (w[i] > 0.0f ? 1.0f : (w[i] < 0.0f ? -1.0f : 0.0f)) * s;
        float d = w[i] - q;
        float d2 = d * d;
        acc = acc + d2;
    }
    return acc;
}

/* window search over [c-2, c+2] -- block_fp2_emu.py:109-131.
 * Keeps the reference's initialisation: best starts at c while best_err starts
 * at the error of the first candidate clamp(c-2), so a strict minimum at c-2
 * still returns c. */
SPO_API int spo_spfp2_search(const float* w8) {
    float maxv = amax_clamp(w8, 8, 1e-38f);
    int c = spo_spfp2_center(maxv);
    int best = c;
    float best_err = 0.0f;
    for (int off = -2; off <= 2; ++off) {
        int e = c + off;
        e = e < 0 ? 0 : (e > 15 ? 15 : e);
        float err = spfp2_err8(w8, e);
        if (off == -2) {
            best_err = err;
        } else if (err < best_err) {
            best = e;
            best_err = err;
        }
    }
    return best;
}

/* mantissa codes for the chosen exponent -- block_fp2_emu.py:39-46
 * code 0: w > s/2 (+1), 1: w < -s/2 (-1), 2: otherwise (0) */
static uint16_t spfp2_mword(const float* w8, int e) {
    const float half = spfp2_scale(e) * 0.5f;
    uint32_t m = 0;
    for (int i = 0; i < 8; ++i) {
        uint32_t code = 2u;
        if (w8[i] > half) code = 0u;
        if (w8[i] < -half) code = 1u;
        m |= code << (2 * i);
    }
    return (uint16_t)m;
}

/* pack_blockwise_search(w, window=2) -- block_fp2_emu.py:86-167
 * out3: nb*3 bytes [m lo, m hi, e]; expv: nb bytes */
SPO_API void spo_spfp2_pack3(const float* w, int64_t n, uint8_t* out3, uint8_t* expv) {
    int64_t nb = n / 8;
    for (int64_t b = 0; b < nb; ++b) {
        const float* wb = w + b * 8;
        int e = spo_spfp2_search(wb);
        uint16_t m = spfp2_mword(wb, e);
        out3[3 * b + 0] = (uint8_t)(m & 0xff);
        out3[3 * b + 1] = (uint8_t)(m >> 8);
        out3[3 * b + 2] = (uint8_t)(e & 0x0f);
        if (expv) expv[b] = (uint8_t)(e & 0x0f);
    }
}

/* pack_blockwise_paired -- block_fp2_emu.py:231-267
 * pair j = blocks (2j, 2j+1): [m0 lo, m0 hi, m1 lo, m1 hi, e0 | e1<<4];
 * an odd block count is padded with an all-zero block (m=0, e=0). */
SPO_API void spo_spfp2_pack_paired(const float* w, int64_t n, uint8_t* out5, uint8_t* expv) {
    int64_t nb = n / 8;
    int64_t np = (nb + 1) / 2;
    for (int64_t p = 0; p < np; ++p) {
        uint16_t m[2] = {0, 0};
        int e[2] = {0, 0};
        for (int h = 0; h < 2; ++h) {
            int64_t b = 2 * p + h;
            if (b >= nb) break;
            const float* wb = w + b * 8;
            e[h] = spo_spfp2_search(wb);
            m[h] = spfp2_mword(wb, e[h]);
            if (expv) expv[b] = (uint8_t)e[h];
        }
        uint8_t* o = out5 + 5 * p;
        o[0] = (uint8_t)(m[0] & 0xff);
        o[1] = (uint8_t)(m[0] >> 8);
        o[2] = (uint8_t)(m[1] & 0xff);
        o[3] = (uint8_t)(m[1] >> 8);
        o[4] = (uint8_t)((e[0] & 0xf) | ((e[1] & 0xf) << 4));
    }
}

/* decode of one block: table (+1,-1,0,0) * 2^(e-10) -- block_fp2_emu.py:36, :216-220 */
static inline void spfp2_decode8(uint16_t m, int e, float* out) {
    const float s = spfp2_scale(e);
    for (int i = 0; i < 8; ++i) {
        uint32_t code = (m >> (2 * i)) & 3u;
        float t = code == 0 ? 1.0f : (code == 1 ? -1.0f : 0.0f);
        out[i] = t * s;
    }
}

/* unpack_blockwise (3-byte) -- block_fp2_emu.py:204-221 */
SPO_API void spo_spfp2_unpack3(const uint8_t* p3, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        uint16_t m = (uint16_t)(p3[3 * b] | (p3[3 * b + 1] << 8));
        spfp2_decode8(m, p3[3 * b + 2] & 0x0f, out + 8 * b);
    }
}

/* Legacy single-exponent blocks of the reference's decode_fp32 / decode_fp16 ops --
 * block_fp2_kernel.cu:3-34: 5 bytes per 16 weights, a little-endian 32-bit word of
 * 2-bit codes and the exponent in the low nibble of byte 4; value = (+1, -1, 0, 0)[code]
 * * 2^(e-10).  The reference forms the scale with __powf(2, e - 10); this restatement
 * takes it as the exact power of two (parity unpinned: that kernel is built for
 * sm_120 and has no golden vectors). */
SPO_API void spo_spfp2_legacy_decode(const uint8_t* p5, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* q = p5 + 5 * b;
        spfp2_decode8((uint16_t)(q[0] | (q[1] << 8)), q[4] & 0x0f, out + 16 * b);
        spfp2_decode8((uint16_t)(q[2] | (q[3] << 8)), q[4] & 0x0f, out + 16 * b + 8);
    }
}

/* unpack_blockwise_paired -- block_fp2_emu.py:270-308 (truncated to n_elements) */
SPO_API void spo_spfp2_unpack_paired(const uint8_t* p5, int64_t n_pairs, int64_t n_elements, float* out) {
    float tmp[16];
    for (int64_t p = 0; p < n_pairs; ++p) {
        const uint8_t* q = p5 + 5 * p;
        uint16_t m0 = (uint16_t)(q[0] | (q[1] << 8));
        uint16_t m1 = (uint16_t)(q[2] | (q[3] << 8));
        spfp2_decode8(m0, q[4] & 0x0f, tmp);
        spfp2_decode8(m1, (q[4] >> 4) & 0x0f, tmp + 8);
        for (int i = 0; i < 16; ++i) {
            int64_t idx = p * 16 + i;
            if (idx < n_elements) out[idx] = tmp[i];
        }
    }
}

/* channel_fake_quantize forward (no-grad path) -- block_fp2_emu.py:365-375:
 * window search over the flattened tensor in 8-blocks, then 3-byte decode */
SPO_API void spo_spfp2_fake_quant(const float* w, int64_t n, float* out) {
    int64_t nb = n / 8;
    for (int64_t b = 0; b < nb; ++b) {
        int e = spo_spfp2_search(w + 8 * b);
        uint16_t m = spfp2_mword(w + 8 * b, e);
        spfp2_decode8(m, e, out + 8 * b);
    }
}

/* ------------------------------------------------------------------------ */
/* float8_e4m3fn                                                             */
/* ------------------------------------------------------------------------ */
/* Round-to-nearest-even conversion to e4m3fn (bias 7, no infinities, 0x7f   */
/* and 0xff are NaN, largest finite 448).  Values whose rounded magnitude    */
/* would exceed 448 (|x| > 464; exactly 464 ties to even 448) become NaN     */
/* with the input's sign, as torch's .to(torch.float8_e4m3fn) does.          */
SPO_API uint8_t spo_f32_to_e4m3(float x) {
    uint32_t u = f2u(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint8_t)(sign | 0x7f);          /* NaN */
    if (a >= 0x43f00000u) return (uint8_t)(sign | 0x7f);         /* >= 480 (and inf) */
    if (a < 0x3c800000u) {                                        /* < 2^-6: subnormal grid 2^-9 */
        /* value / 2^-9 rounded half-even, 0..8 (8 == smallest normal) */
        float v = u2f(a) * 512.0f;                                /* exact scaling */
        float r = rintf(v);                                       /* default mode: RNE */
        return (uint8_t)(sign | (uint8_t)r);
    }
    int exp = (int)(a >> 23) - 127;                               /* -6 .. 8 */
    uint32_t mant = a & 0x7fffffu;
    uint32_t keep = mant >> 20;                                   /* 3 bits */
    uint32_t rest = mant & 0xfffffu;
    uint32_t halfway = 0x80000u;
    if (rest > halfway || (rest == halfway && (keep & 1u))) {
        keep += 1;
        if (keep == 8) { keep = 0; exp += 1; }
    }
    uint32_t code = ((uint32_t)(exp + 7) << 3) | keep;            /* exp <= 8 here, code <= 0x7e */
    if (code >= 0x7f) return (uint8_t)(sign | 0x7f);
    return (uint8_t)(sign | code);
}

SPO_API float spo_e4m3_to_f32(uint8_t b) {
    uint32_t sign = (uint32_t)(b & 0x80) << 24;
    uint32_t e = (b >> 3) & 0xf, m = b & 7;
    if (e == 0xf && m == 7) return u2f(sign | 0x7ff00000u);          /* torch's NaN bits */
    if (e == 0) {
        float v = (float)m * (1.0f / 512.0f);
        return sign ? -v : v;
    }
    return u2f(sign | ((e + 120) << 23) | (m << 20));
}

/* ------------------------------------------------------------------------ */
/* FP3 E1M1 -- fp3_emu.py                                                    */
/* ------------------------------------------------------------------------ */
static const float FP3_TABLE[8] = {0.0f, 0.5f, 1.0f, 1.5f, -0.0f, -0.5f, -1.0f, -1.5f}; /* :47 */

/* quantise one padded 16-block: scale byte + 16 codes -- fp3_emu.py:107-126 */
static void fp3_quant16(const float* w16, uint8_t* scale8, uint8_t* codes) {
    float amax = amax_clamp(w16, 16, 0.0f);
    float sf = amax / 1.5f;
    if (!(sf >= 1e-30f) && !isnan(sf)) sf = 1e-30f;               /* clamp_min(1e-30) */
    uint8_t s8 = spo_f32_to_e4m3(sf);
    float s = spo_e4m3_to_f32(s8);
    *scale8 = s8;
    for (int i = 0; i < 16; ++i) {
        float xs = w16[i] / s;
        float ax = fabsf(xs);
        int mag = isnan(ax) ? 3 : (ax > 0.25f) + (ax > 0.75f) + (ax > 1.25f);
        int sg = xs < 0.0f;
        codes[i] = (uint8_t)((sg << 2) | mag);
    }
}

/* row-padded code/scale generation shared by all FP3 packers */
static void fp3_quant_matrix(const float* w, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales) {
    int64_t nb = (ic + 15) / 16;
    float blk[16];
    for (int64_t r = 0; r < oc; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            for (int i = 0; i < 16; ++i) {
                int64_t c = b * 16 + i;
                blk[i] = c < ic ? w[r * ic + c] : 0.0f;
            }
            fp3_quant16(blk, scales + r * nb + b, codes + (r * nb + b) * 16);
        }
}

/* fp3_pack_3bit -- fp3_emu.py:107-139: codes (oc*nb*16, padded to 8) in
 * 24-bit LE groups, code i of a group at bits 3i.  codes buffer is scratch. */
SPO_API void spo_fp3_pack3bit(const float* w, int64_t oc, int64_t ic, uint8_t* packed, uint8_t* scales) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)calloc((size_t)(n + 8), 1);
    fp3_quant_matrix(w, oc, ic, codes, scales);
    int64_t ng = (n + 7) / 8;
    for (int64_t g = 0; g < ng; ++g) {
        uint32_t v = 0;
        for (int i = 0; i < 8; ++i) v |= (uint32_t)codes[g * 8 + i] << (3 * i);
        packed[3 * g + 0] = (uint8_t)(v & 0xff);
        packed[3 * g + 1] = (uint8_t)((v >> 8) & 0xff);
        packed[3 * g + 2] = (uint8_t)((v >> 16) & 0xff);
    }
    free(codes);
}

/* fp3_pack (nibble) -- fp3_emu.py:50-73 */
SPO_API void spo_fp3_pack_nibble(const float* w, int64_t oc, int64_t ic, uint8_t* packed, uint8_t* scales) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)calloc((size_t)(n + 2), 1);
    fp3_quant_matrix(w, oc, ic, codes, scales);
    for (int64_t j = 0; j < (n + 1) / 2; ++j)
        packed[j] = (uint8_t)((codes[2 * j] & 0xf) | ((codes[2 * j + 1] & 0xf) << 4));
    free(codes);
}

static void fp3_expand(const uint8_t* codes, const uint8_t* scales, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    for (int64_t r = 0; r < oc; ++r)
        for (int64_t c = 0; c < ic; ++c) {
            int64_t k = r * nb * 16 + c;
            float s = spo_e4m3_to_f32(scales[k / 16]);
            out[r * ic + c] = FP3_TABLE[codes[k] & 7] * s;
        }
}

/* fp3_unpack_3bit -- fp3_emu.py:142-154 */
SPO_API void spo_fp3_unpack3bit(const uint8_t* packed, const uint8_t* scales, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)malloc((size_t)n);
    for (int64_t k = 0; k < n; ++k) {
        int64_t g = k / 8;
        uint32_t v = packed[3 * g] | (packed[3 * g + 1] << 8) | (packed[3 * g + 2] << 16);
        codes[k] = (uint8_t)((v >> (3 * (k % 8))) & 7u);
    }
    fp3_expand(codes, scales, oc, ic, out);
    free(codes);
}

/* fp3_unpack (nibble) -- fp3_emu.py:76-86 (code & 0xF clamped to 7) */
SPO_API void spo_fp3_unpack_nibble(const uint8_t* packed, const uint8_t* scales, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)malloc((size_t)n);
    for (int64_t k = 0; k < n; ++k) {
        uint8_t nib = (k & 1) ? (packed[k / 2] >> 4) : (packed[k / 2] & 0xf);
        codes[k] = nib > 7 ? 7 : nib;
    }
    fp3_expand(codes, scales, oc, ic, out);
    free(codes);
}

/* fp3_fake_quant -- fp3_emu.py:24-43 */
SPO_API void spo_fp3_fake_quant(const float* w, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)malloc((size_t)n);
    uint8_t* scales = (uint8_t*)malloc((size_t)(oc * nb));
    fp3_quant_matrix(w, oc, ic, codes, scales);
    fp3_expand(codes, scales, oc, ic, out);
    free(codes);
    free(scales);
}

/* ------------------------------------------------------------------------ */
/* NVFP4 -- nvfp4_emu.py                                                     */
/* ------------------------------------------------------------------------ */
static const float E2M1_POS[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f}; /* :20 */
static const float E2M1_BOUNDS[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f}; /* :22 */

static inline int e2m1_bucket(float ax) {
    if (isnan(ax)) return 7;
    int idx = 0;
    for (int i = 0; i < 7; ++i) idx += ax > E2M1_BOUNDS[i];
    return idx;
}

/* per 16-block: scale = fp8(clamp_min(amax/6, 1e-30)) -- nvfp4_emu.py:92-96 */
static uint8_t nvfp4_scale16(const float* w16, float* s_out) {
    float amax = amax_clamp(w16, 16, 0.0f);
    float sf = amax / 6.0f;
    if (!(sf >= 1e-30f) && !isnan(sf)) sf = 1e-30f;
    uint8_t s8 = spo_f32_to_e4m3(sf);
    *s_out = spo_e4m3_to_f32(s8);
    return s8;
}

static void nvfp4_codes_matrix(const float* w, int64_t oc, int64_t ic, uint8_t* codes, uint8_t* scales) {
    int64_t nb = (ic + 15) / 16;
    float blk[16];
    for (int64_t r = 0; r < oc; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            for (int i = 0; i < 16; ++i) {
                int64_t c = b * 16 + i;
                blk[i] = c < ic ? w[r * ic + c] : 0.0f;
            }
            float s;
            scales[r * nb + b] = nvfp4_scale16(blk, &s);
            for (int i = 0; i < 16; ++i) {
                float xs = blk[i] / s;
                int idx = e2m1_bucket(fabsf(xs));
                codes[(r * nb + b) * 16 + i] = (uint8_t)(idx + (xs < 0.0f ? 8 : 0));
            }
        }
}

/* nvfp4_pack -- nvfp4_emu.py:81-107 (element 2j low nibble, 2j+1 high) */
SPO_API void spo_nvfp4_pack(const float* w, int64_t oc, int64_t ic, uint8_t* packed, uint8_t* scales) {
    int64_t nb = (ic + 15) / 16;
    int64_t n = oc * nb * 16;
    uint8_t* codes = (uint8_t*)calloc((size_t)(n + 2), 1);
    nvfp4_codes_matrix(w, oc, ic, codes, scales);
    for (int64_t j = 0; j < (n + 1) / 2; ++j)
        packed[j] = (uint8_t)((codes[2 * j] & 0xf) | ((codes[2 * j + 1] & 0xf) << 4));
    free(codes);
}

/* nvfp4_unpack -- nvfp4_emu.py:109-123 */
SPO_API void spo_nvfp4_unpack(const uint8_t* packed, const uint8_t* scales, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    for (int64_t r = 0; r < oc; ++r)
        for (int64_t c = 0; c < ic; ++c) {
            int64_t k = r * nb * 16 + c;
            uint8_t code = (k & 1) ? (packed[k / 2] >> 4) : (packed[k / 2] & 0xf);
            float v = code < 8 ? E2M1_POS[code] : -E2M1_POS[code - 8];
            out[r * ic + c] = v * spo_e4m3_to_f32(scales[k / 16]);
        }
}

/* nvfp4_fake_quant -- nvfp4_emu.py:37-57: sign(x) * q, with sign(NaN) = 0 */
SPO_API void spo_nvfp4_fake_quant(const float* w, int64_t oc, int64_t ic, float* out) {
    int64_t nb = (ic + 15) / 16;
    float blk[16];
    for (int64_t r = 0; r < oc; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            for (int i = 0; i < 16; ++i) {
                int64_t c = b * 16 + i;
                blk[i] = c < ic ? w[r * ic + c] : 0.0f;
            }
            float s;
            nvfp4_scale16(blk, &s);
            for (int i = 0; i < 16; ++i) {
                int64_t c = b * 16 + i;
                if (c >= ic) break;
                float xs = blk[i] / s;
                float q = E2M1_POS[e2m1_bucket(fabsf(xs))];
                float sg = xs > 0.0f ? 1.0f : (xs < 0.0f ? -1.0f : 0.0f);
                out[r * ic + c] = (sg * q) * s;
            }
        }
}

/* ------------------------------------------------------------------------ */
/* 2:4-sparse SPFP2 -- two_four.py                                           */
/* ------------------------------------------------------------------------ */
static const int TF_DUAL[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}}; /* :23 */

static int tf_dual_index(int a, int b) {
    for (int i = 0; i < 6; ++i)
        if (TF_DUAL[i][0] == a && TF_DUAL[i][1] == b) return i;
    return 0;
}

/* err of a 16-block: lanes k and k+8 summed first, then lanes 0..7 in order
 * (torch full-tensor sum) -- two_four.py:105-106 */
static float tf_err16(const float* w, int e) {
    const float s = spfp2_scale(e);
    const float half = s * 0.5f;
    float d2[16];
    for (int i = 0; i < 16; ++i) {
        float q = 0.0f;
        if (fabsf(w[i]) > half) q = (w[i] > 0.0f ? 1.0f : (w[i] < 0.0f ? -1.0f : 0.0f)) * s;
        float d = w[i] - q;
        d2[i] = d * d;
    }
    float acc = 0.0f;
    for (int k = 0; k < 8; ++k) {
        float l = d2[k] + d2[k + 8];
        acc = acc + l;
    }
    return acc;
}

/* _search_exp -- two_four.py:98-109 (first candidate always accepted) */
SPO_API int spo_twofour_search(const float* w16) {
    float maxv = amax_clamp(w16, 16, 1e-38f);
    int c = spo_spfp2_center(maxv);
    int best = 0;
    float best_err = 0.0f;
    for (int off = -2; off <= 2; ++off) {
        int e = c + off;
        e = e < 0 ? 0 : (e > 15 ? 15 : e);
        float err = tf_err16(w16, e);
        if (off == -2 || err < best_err) {
            best = e;
            best_err = err;
        }
    }
    return best;
}

/* ternary value of w at exponent e: +1, -1 or 0 -- two_four.py:90-95 */
static inline int tf_tern(float w, float half) {
    if (fabsf(w) > half) return w > 0.0f ? 1 : (w < 0.0f ? -1 : 0);
    return 0;
}

/* 28-bit slot code of one 16-block -- two_four.py:136-147 */
static uint32_t tf_encode16(const float* w16, int e) {
    const float half = spfp2_scale(e) * 0.5f;
    uint32_t v = 0;
    for (int g = 0; g < 4; ++g) {
        int t[4], nz[4], cnt = 0;
        for (int i = 0; i < 4; ++i) {
            t[i] = tf_tern(w16[4 * g + i], half);
            if (t[i] != 0) nz[cnt++] = i;
        }
        /* two_four_apply keeps the first two nonzeros (stable sort on |q|) */
        uint32_t mode, s0 = 0, s1 = 0;
        if (cnt == 0) {
            mode = 15;
        } else if (cnt == 1) {
            mode = 8 + nz[0];
            s0 = t[nz[0]] < 0;
        } else {
            mode = tf_dual_index(nz[0], nz[1]);
            s0 = t[nz[0]] < 0;
            s1 = t[nz[1]] < 0;
        }
        v |= mode << (4 * g);
        v |= s0 << (16 + 2 * g);
        v |= s1 << (16 + 2 * g + 1);
    }
    v |= (uint32_t)(e & 0xf) << 24;
    return v;
}

/* two_four_pack -- two_four.py:112-155.  Rows padded to 16 columns, the
 * flattened 16-block count padded to even; 7 LE bytes per pair of blocks. */
SPO_API void spo_twofour_pack(const float* w, int64_t oc, int64_t ic, uint8_t* out) {
    int64_t nb_ic = (ic + 15) / 16;
    int64_t nb = oc * nb_ic;
    int64_t np = (nb + 1) / 2;
    float blk[16];
    for (int64_t p = 0; p < np; ++p) {
        uint64_t v = 0;
        for (int h = 0; h < 2; ++h) {
            int64_t b = 2 * p + h;
            if (b < nb) {
                int64_t r = b / nb_ic, cb = b % nb_ic;
                for (int i = 0; i < 16; ++i) {
                    int64_t c = cb * 16 + i;
                    blk[i] = c < ic ? w[r * ic + c] : 0.0f;
                }
            } else {
                memset(blk, 0, sizeof(blk));
            }
            int e = spo_twofour_search(blk);
            v |= (uint64_t)tf_encode16(blk, e) << (28 * h);
        }
        for (int k = 0; k < 7; ++k) out[7 * p + k] = (uint8_t)((v >> (8 * k)) & 0xff);
    }
}

/* two_four_unpack -- two_four.py:158-189 */
SPO_API void spo_twofour_unpack(const uint8_t* packed, int64_t n_pairs, int64_t n_elements, float* out) {
    for (int64_t p = 0; p < n_pairs; ++p) {
        uint64_t v = 0;
        for (int k = 0; k < 7; ++k) v |= (uint64_t)packed[7 * p + k] << (8 * k);
        for (int slot = 0; slot < 2; ++slot) {
            uint32_t w = (uint32_t)(v >> (28 * slot)) & 0x0fffffffu;
            float s = spfp2_scale((w >> 24) & 0xf);
            for (int g = 0; g < 4; ++g) {
                int mode = (w >> (4 * g)) & 0xf;
                int s0 = (w >> (16 + 2 * g)) & 1, s1 = (w >> (17 + 2 * g)) & 1;
                float vals[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (mode < 6) {
                    vals[TF_DUAL[mode][0]] = s0 ? -s : s;
                    vals[TF_DUAL[mode][1]] = s1 ? -s : s;
                } else if (mode >= 8 && mode <= 11) {
                    vals[mode - 8] = s0 ? -s : s;
                }
                for (int i = 0; i < 4; ++i) {
                    int64_t idx = p * 32 + slot * 16 + g * 4 + i;
                    if (idx < n_elements) out[idx] = vals[i];
                }
            }
        }
    }
}

/* two_four_fake_quant -- two_four.py:70-75: channel_fake_quantize over the
 * flattened tensor, then two_four_apply on flattened groups of 4 (the first
 * two nonzeros survive; dropped values are multiplied by 0.0, so a dropped
 * negative becomes -0.0). */
SPO_API void spo_twofour_fake_quant(const float* w, int64_t n, float* out) {
    spo_spfp2_fake_quant(w, n, out);
    for (int64_t g = 0; g < n / 4; ++g) {
        int kept = 0;
        for (int i = 0; i < 4; ++i) {
            float* v = out + 4 * g + i;
            if (*v != 0.0f) {
                if (kept < 2) kept++;
                else *v = *v * 0.0f;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* linear references                                                         */
/* ------------------------------------------------------------------------ */
/* y[M, oc] = x[M, ic] . W[oc, ic]^T (+ bias), fp64 accumulation: the ground
 * truth the GEMV/GEMM tolerances are stated against. */
SPO_API void spo_linear_f64(const float* x, int64_t M, int64_t ic, const float* W, int64_t oc,
                            const float* bias, double* y) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t r = 0; r < oc; ++r) {
            double acc = bias ? (double)bias[r] : 0.0;
            const float* wr = W + r * ic;
            const float* xm = x + m * ic;
            for (int64_t k = 0; k < ic; ++k) acc += (double)xm[k] * (double)wr[k];
            y[m * oc + r] = acc;
        }
}

SPO_API int spo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the OpenMP regions below (launchers such as torchrun set
 * OMP_NUM_THREADS=1 per process; the CPU baseline sets it explicitly). */
SPO_API void spo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* CPU baseline of the reference's online path (decode + fp32 matmul per
 * call, the arithmetic of unpack_blockwise_paired followed by
 * x.float() @ W.T): one SPFP2 paired linear, rows split across threads. */
SPO_API void spo_cpu_spfp2_linear(const uint8_t* p5, const float* x, int64_t M, int64_t oc, int64_t ic,
                                  float* y) {
    int64_t pairs_per_row = ic / 16;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < oc; ++r) {
        float wrow[16];
        float acc[64];
        int64_t mm = M < 64 ? M : 64;
        for (int64_t m = 0; m < mm; ++m) acc[m] = 0.0f;
        for (int64_t p = 0; p < pairs_per_row; ++p) {
            const uint8_t* q = p5 + 5 * (r * pairs_per_row + p);
            spfp2_decode8((uint16_t)(q[0] | (q[1] << 8)), q[4] & 0xf, wrow);
            spfp2_decode8((uint16_t)(q[2] | (q[3] << 8)), (q[4] >> 4) & 0xf, wrow + 8);
            for (int64_t m = 0; m < mm; ++m) {
                const float* xm = x + m * ic + p * 16;
                float a = acc[m];
                for (int i = 0; i < 16; ++i) a += xm[i] * wrow[i];
                acc[m] = a;
            }
        }
        for (int64_t m = 0; m < mm; ++m) y[m * oc + r] = acc[m];
    }
}

/* Same for FP3 (3-bit codes + e4m3 scales, ic % 16 == 0). */
SPO_API void spo_cpu_fp3_linear(const uint8_t* codes, const uint8_t* scales, const float* x, int64_t M,
                                int64_t oc, int64_t ic, float* y) {
    int64_t nb = ic / 16;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < oc; ++r) {
        float acc[64];
        int64_t mm = M < 64 ? M : 64;
        for (int64_t m = 0; m < mm; ++m) acc[m] = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            float wv[16];
            float s = spo_e4m3_to_f32(scales[r * nb + b]);
            const uint8_t* g = codes + (r * nb + b) * 6;
            uint32_t v0 = g[0] | (g[1] << 8) | (g[2] << 16);
            uint32_t v1 = g[3] | (g[4] << 8) | (g[5] << 16);
            for (int i = 0; i < 8; ++i) wv[i] = FP3_TABLE[(v0 >> (3 * i)) & 7] * s;
            for (int i = 0; i < 8; ++i) wv[8 + i] = FP3_TABLE[(v1 >> (3 * i)) & 7] * s;
            for (int64_t m = 0; m < mm; ++m) {
                const float* xm = x + m * ic + b * 16;
                float a = acc[m];
                for (int i = 0; i < 16; ++i) a += xm[i] * wv[i];
                acc[m] = a;
            }
        }
        for (int64_t m = 0; m < mm; ++m) y[m * oc + r] = acc[m];
    }
}

/* Same for NVFP4 (nibble codes + e4m3 scales, ic % 16 == 0). */
SPO_API void spo_cpu_nvfp4_linear(const uint8_t* codes, const uint8_t* scales, const float* x, int64_t M,
                                  int64_t oc, int64_t ic, float* y) {
    int64_t nb = ic / 16;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < oc; ++r) {
        float acc[64];
        int64_t mm = M < 64 ? M : 64;
        for (int64_t m = 0; m < mm; ++m) acc[m] = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            float wv[16];
            float s = spo_e4m3_to_f32(scales[r * nb + b]);
            const uint8_t* g = codes + (r * nb + b) * 8;
            for (int i = 0; i < 16; ++i) {
                uint8_t c = (i & 1) ? (g[i / 2] >> 4) : (g[i / 2] & 0xf);
                wv[i] = (c < 8 ? E2M1_POS[c] : -E2M1_POS[c - 8]) * s;
            }
            for (int64_t m = 0; m < mm; ++m) {
                const float* xm = x + m * ic + b * 16;
                float a = acc[m];
                for (int i = 0; i < 16; ++i) a += xm[i] * wv[i];
                acc[m] = a;
            }
        }
        for (int64_t m = 0; m < mm; ++m) y[m * oc + r] = acc[m];
    }
}

/* ------------------------------------------------------------------------ */
/* per-channel symmetric INT8 -- int8_emu.py                                 */
/* ------------------------------------------------------------------------ */
/* int8_emu.py:15 / :43: scale = (|w|.amax(dim=1) / 127).clamp_min(1e-12); a NaN
 * in the row makes amax (and the scale) NaN, as torch.amax propagates NaN. */
static float int8_scale(const float* row, int64_t ic) {
    float amax = 0.0f;
    int nan = 0;
    for (int64_t c = 0; c < ic; ++c) {
        float a = fabsf(row[c]);
        if (a != a) nan = 1;
        else if (a > amax) amax = a;
    }
    if (nan) return NAN;
    float s = amax / 127.0f;
    return s < 1e-12f ? 1e-12f : s;
}

/* :16 / :44: torch.round (half to even) of w / scale, clamp to +-127 (NaN stays) */
static float int8_q(float v, float s) {
    float q = nearbyintf(v / s);
    return q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
}

/* int8_fake_quant -- int8_emu.py:12-18 */
SPO_API void spo_int8_fake_quant(const float* w, int64_t oc, int64_t ic, float* out) {
    for (int64_t r = 0; r < oc; ++r) {
        float s = int8_scale(w + r * ic, ic);
        for (int64_t c = 0; c < ic; ++c) out[r * ic + c] = int8_q(w[r * ic + c], s) * s;
    }
}

/* ptq_int8_pack -- int8_emu.py:37-46 (rows without NaN) */
SPO_API void spo_int8_pack(const float* w, int64_t oc, int64_t ic, int8_t* q, float* scale) {
    for (int64_t r = 0; r < oc; ++r) {
        float s = int8_scale(w + r * ic, ic);
        scale[r] = s;
        for (int64_t c = 0; c < ic; ++c) q[r * ic + c] = (int8_t)(int)int8_q(w[r * ic + c], s);
    }
}
