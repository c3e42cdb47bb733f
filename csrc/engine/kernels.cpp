// FP4 row-dot kernels (see kernels.h). Each ISA's functions carry a target attribute, so one library holds all of them
// and the engine picks the best one the CPU supports at run time (XTIER_ISA overrides).
#include "kernels.h"

#include <immintrin.h>
#include <math.h>
#include <string.h>

namespace xt {

static const float kE2M1[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f, -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

float e4m3_value(uint8_t b) {
    int e = (b >> 3) & 0xF, m = b & 7;
    float v = e ? ldexpf(1.f + m / 8.f, e - 7) : ldexpf(m / 8.f, -6);
    return (b & 0x80) ? -v : v;
}

float ue8m0_value(uint8_t b) { return ldexpf(1.f, int(b) - 127); }

static float bf16_to_f32(uint16_t h) {
    uint32_t u = uint32_t(h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);   // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}

static inline float block_scale(const uint8_t *s, int k, int fmt) {
    return fmt == NVFP4 ? e4m3_value(s[k >> 4]) : ue8m0_value(s[k >> 5]);
}

// ---------------------------------------------------------------- scalar
static void prep_x_scalar(const uint16_t *x, int K, void *dst) {
    float *d = static_cast<float *>(dst);
    for (int k = 0; k < K; ++k) d[k] = bf16_to_f32(x[k]);
}

static void store_mid_scalar(void *dst, int, int j, float v) { static_cast<float *>(dst)[j] = v; }

static void dot_scalar(const uint8_t *w, size_t ws, const uint8_t *s, size_t ss, int rows, int K, int fmt,
                       const void *const *xs, int n, int, float *out) {
    const int bs = fmt == NVFP4 ? 16 : 32;
    for (int r = 0; r < rows; ++r) {
        const uint8_t *wr = w + r * ws, *sr = s + r * ss;
        for (int t = 0; t < n; ++t) {
            const float *x = static_cast<const float *>(xs[t]);
            float acc = 0.f;
            for (int b = 0; b < K / bs; ++b) {
                float part = 0.f;
                for (int i = 0; i < bs; i += 2) {
                    uint8_t byte = wr[(b * bs + i) >> 1];
                    part += kE2M1[byte & 15] * x[b * bs + i] + kE2M1[byte >> 4] * x[b * bs + i + 1];
                }
                acc += part * block_scale(sr, b * bs, fmt);
            }
            out[r * n + t] = acc;
        }
    }
}

static const Kernels kScalar = {"scalar", 32, 4, 4, prep_x_scalar, store_mid_scalar, dot_scalar};
const Kernels *kernels_scalar() { return &kScalar; }

// ---------------------------------------------------------------- AVX2 + FMA (FP32 arithmetic)
#define XT_AVX2 __attribute__((target("avx2,fma")))

XT_AVX2 static void prep_x_avx2(const uint16_t *x, int K, void *dst) {
    float *d = static_cast<float *>(dst);
    for (int c = 0; c < K; c += 16)
        for (int i = 0; i < 8; ++i) {
            d[c + i] = bf16_to_f32(x[c + 2 * i]);
            d[c + 8 + i] = bf16_to_f32(x[c + 2 * i + 1]);
        }
}

static void store_mid_avx2(void *dst, int, int j, float v) {
    int c = j & ~15, i = j & 15;
    static_cast<float *>(dst)[c + (i & 1) * 8 + (i >> 1)] = v;
}

XT_AVX2 static inline __m256 fp4_decode8(__m256i codes, __m256 lut) {
    __m256 mag = _mm256_permutevar8x32_ps(lut, codes);   // uses the low 3 bits
    __m256i sign = _mm256_slli_epi32(_mm256_and_si256(codes, _mm256_set1_epi32(8)), 28);
    return _mm256_xor_ps(mag, _mm256_castsi256_ps(sign));
}

XT_AVX2 static void dot_avx2(const uint8_t *w, size_t ws, const uint8_t *s, size_t ss, int rows, int K, int fmt,
                             const void *const *xs, int n, int, float *out) {
    const __m256 lut = _mm256_setr_ps(0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f);
    const __m256i m15 = _mm256_set1_epi32(15);
    for (int r = 0; r < rows; ++r) {
        const uint8_t *wr = w + r * ws, *sr = s + r * ss;
        __m256 acc[MAX_TOK];
        for (int t = 0; t < n; ++t) acc[t] = _mm256_setzero_ps();
        for (int c = 0; c < K; c += 16) {
            long long v;
            memcpy(&v, wr + c / 2, 8);
            __m256i b = _mm256_cvtepu8_epi32(_mm_cvtsi64_si128(v));
            __m256 we = fp4_decode8(_mm256_and_si256(b, m15), lut);
            __m256 wo = fp4_decode8(_mm256_srli_epi32(b, 4), lut);
            __m256 sc = _mm256_set1_ps(block_scale(sr, c, fmt));
            for (int t = 0; t < n; ++t) {
                const float *x = static_cast<const float *>(xs[t]) + c;
                __m256 d = _mm256_mul_ps(we, _mm256_loadu_ps(x));
                d = _mm256_fmadd_ps(wo, _mm256_loadu_ps(x + 8), d);
                acc[t] = _mm256_fmadd_ps(d, sc, acc[t]);
            }
        }
        for (int t = 0; t < n; ++t) {
            __m128 h = _mm_add_ps(_mm256_castps256_ps128(acc[t]), _mm256_extractf128_ps(acc[t], 1));
            h = _mm_add_ps(h, _mm_movehl_ps(h, h));
            h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 1));
            out[r * n + t] = _mm_cvtss_f32(h);
        }
    }
}

static const Kernels kAvx2 = {"avx2", 32, 4, 4, prep_x_avx2, store_mid_avx2, dot_avx2};

// ---------------------------------------------------------------- AVX-512 BF16 (vdpbf16ps on exact BF16 weights)
#define XT_AVX512 __attribute__((target("avx512f,avx512bw,avx512vl,avx512dq,avx512bf16")))

// E2M1 code -> BF16 bits; e2m1 values times E4M3 / UE8M0 scales are exact in FP32, and the code values themselves are
// exact in BF16, so vdpbf16ps products are exact and only the FP32 sums round.
static const uint16_t kE2M1Bf16[32] = {0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0,
                                       0x8000, 0xBF00, 0xBF80, 0xBFC0, 0xC000, 0xC040, 0xC080, 0xC0C0};

XT_AVX512 static void prep_x_avx512(const uint16_t *x, int K, void *dst) {
    uint16_t *d = static_cast<uint16_t *>(dst);
    for (int c = 0; c < K; c += 64)
        for (int i = 0; i < 32; ++i) {
            d[c + i] = x[c + 2 * i];
            d[c + 32 + i] = x[c + 2 * i + 1];
        }
}

// hi chunk layout over all K first, then lo: dst holds 2*K BF16 values
static void store_mid_avx512(void *dst, int K, int j, float v) {
    uint16_t *d = static_cast<uint16_t *>(dst);
    int c = j & ~63, i = j & 63;
    int pos = c + (i & 1) * 32 + (i >> 1);
    uint16_t hi = f32_to_bf16_rne(v);
    d[pos] = hi;
    d[K + pos] = f32_to_bf16_rne(v - bf16_to_f32(hi));
}

// All block scales of one row -> FP32 (16 at a time; the tail of the buffer is padded, never read as a scale).
XT_AVX512 static void row_scales(const uint8_t *sr, int nblocks, int fmt, float *sf) {
    for (int i = 0; i < nblocks; i += 16) {
        const __mmask16 m = nblocks - i >= 16 ? __mmask16(0xFFFF) : __mmask16((1u << (nblocks - i)) - 1);
        const __m512i b = _mm512_cvtepu8_epi32(_mm_maskz_loadu_epi8(m, sr + i));
        __m512 f;
        if (fmt == NVFP4) {
            const __m512i mag = _mm512_and_si512(b, _mm512_set1_epi32(0x7F));
            const __m512 normal =
                _mm512_castsi512_ps(_mm512_add_epi32(_mm512_slli_epi32(mag, 20), _mm512_set1_epi32(120 << 23)));
            const __m512 sub = _mm512_mul_ps(_mm512_cvtepi32_ps(mag), _mm512_set1_ps(0x1p-9f));
            f = _mm512_mask_blend_ps(_mm512_cmplt_epi32_mask(mag, _mm512_set1_epi32(8)), normal, sub);
        } else {
            f = _mm512_castsi512_ps(_mm512_slli_epi32(b, 23));   // exponent byte 0 reads as 0 instead of 2^-127
        }
        _mm512_storeu_ps(sf + i, f);
    }
}

// N tokens (compile time, so the accumulators stay in registers) and HILO (the down projection's hi+lo intermediate)
// are template parameters; two accumulators per token alternate between chunks to halve the FMA dependency chain.
template <int N, bool HILO>
XT_AVX512 static void dot_avx512_n(const uint8_t *w, size_t ws, const uint8_t *s, size_t ss, int rows, int K, int fmt,
                                   const void *const *xs, float *out) {
    const __m512i lut = _mm512_loadu_si512(kE2M1Bf16);
    const __m512i m15 = _mm512_set1_epi16(15);
    // lane l of a 64-element chunk covers elements 4l..4l+3: NVFP4 block l/4, MXFP4 block l/8
    const __m512i rep = fmt == NVFP4 ? _mm512_setr_epi32(0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3)
                                     : _mm512_setr_epi32(0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1);
    const int bs = fmt == NVFP4 ? 16 : 32;
    const int bshift = fmt == NVFP4 ? 4 : 5;   // c / bs without a division in the loop
    alignas(64) float sf[16384 / 16 + 16];
    const uint16_t *x[N];
    for (int t = 0; t < N; ++t) x[t] = static_cast<const uint16_t *>(xs[t]);
    for (int r = 0; r < rows; ++r) {
        const uint8_t *wr = w + r * ws, *sr = s + r * ss;
        row_scales(sr, K / bs, fmt, sf);
        __m512 acc0[N], acc1[N];
#pragma GCC unroll 8
        for (int t = 0; t < N; ++t) acc0[t] = acc1[t] = _mm512_setzero_ps();
#define XT_CHUNK(CC, ACC)                                                                                      \
    {                                                                                                          \
        const int c_ = (CC);                                                                                   \
        __m512i b = _mm512_cvtepu8_epi16(_mm256_loadu_si256(reinterpret_cast<const __m256i *>(wr + c_ / 2)));  \
        __m512bh we = (__m512bh)_mm512_permutexvar_epi16(_mm512_and_si512(b, m15), lut);                       \
        __m512bh wo = (__m512bh)_mm512_permutexvar_epi16(_mm512_srli_epi16(b, 4), lut);                        \
        __m512 sc = _mm512_permutexvar_ps(rep, _mm512_castps128_ps512(_mm_loadu_ps(sf + (c_ >> bshift))));     \
        _Pragma("GCC unroll 8") for (int t = 0; t < N; ++t) {                                                  \
            const uint16_t *xt = x[t] + c_;                                                                    \
            __m512 d = _mm512_dpbf16_ps(_mm512_setzero_ps(), we, (__m512bh)_mm512_loadu_si512(xt));            \
            d = _mm512_dpbf16_ps(d, wo, (__m512bh)_mm512_loadu_si512(xt + 32));                                \
            if (HILO) {                                                                                        \
                d = _mm512_dpbf16_ps(d, we, (__m512bh)_mm512_loadu_si512(xt + K));                             \
                d = _mm512_dpbf16_ps(d, wo, (__m512bh)_mm512_loadu_si512(xt + K + 32));                        \
            }                                                                                                  \
            ACC[t] = _mm512_fmadd_ps(d, sc, ACC[t]);                                                           \
        }                                                                                                      \
    }
        int c = 0;
        for (; c + 128 <= K; c += 128) {
            XT_CHUNK(c, acc0)
            XT_CHUNK(c + 64, acc1)
        }
        if (c < K) XT_CHUNK(c, acc0)
#undef XT_CHUNK
#pragma GCC unroll 8
        for (int t = 0; t < N; ++t) out[r * N + t] = _mm512_reduce_add_ps(_mm512_add_ps(acc0[t], acc1[t]));
    }
}

XT_AVX512 static void dot_avx512(const uint8_t *w, size_t ws, const uint8_t *s, size_t ss, int rows, int K, int fmt,
                                 const void *const *xs, int n, int hilo, float *out) {
#define XT_DOT_N(NN)                                                                                  \
    case NN:                                                                                          \
        return hilo ? dot_avx512_n<NN, true>(w, ws, s, ss, rows, K, fmt, xs, out)                    \
                    : dot_avx512_n<NN, false>(w, ws, s, ss, rows, K, fmt, xs, out);
    switch (n) {
        XT_DOT_N(1) XT_DOT_N(2) XT_DOT_N(3) XT_DOT_N(4) XT_DOT_N(5) XT_DOT_N(6) XT_DOT_N(7) XT_DOT_N(8)
        default: break;
    }
#undef XT_DOT_N
}

static const Kernels kAvx512 = {"avx512", 64, 2, 4, prep_x_avx512, store_mid_avx512, dot_avx512};

const Kernels *kernels_avx512() {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
        __builtin_cpu_supports("avx512bf16"))
        return &kAvx512;
    return nullptr;
}

const Kernels *kernels_avx2() {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return &kAvx2;
    return nullptr;
}

}  // namespace xt
