// Model-pack kernels of the DeepSeek V4 and Qwen4-exp families, as standalone ops:
//
// mhc_post   the manifold hyper-connection post-mix of DeepSeek V4: out[m, i, :] = BF16(post[m, i] * x[m, :] +
//            (((comb[m, 0, i] * res[m, 0, :] + comb[m, 1, i] * res[m, 1, :]) + comb[m, 2, i] * res[m, 2, :]) +
//            comb[m, 3, i] * res[m, 3, :])), every product and sum rounded to nearest in FP32 in exactly this order
//            (no fused multiply-add), so the result is bit-identical to the same expression evaluated by PyTorch; one
//            thread per 8 columns of one row, all four outputs from one read of x and the four residual streams.
//            Reference: xtier/packs/deepseek_v4/mhc_sm120.py:31-92 (the same expression and order).
// wo_a       DeepSeek V4's grouped low-rank attention output projection at decode sizes: out[t, g, r] =
//            sum_h o[t, g, h] * W[g, r, h] with W in FP8 E4M3 and one FP32 (power-of-two) scale per 32 x 32 block
//            of the [G * R, D] weight, or W in BF16; FP32 accumulation. One CTA per (group, 32 weight rows): the
//            weight streams once through 16-byte loads, the tokens' activations of the group through shared memory in
//            256-column chunks, up to 16 tokens per pass. Reference: xtier/packs/deepseek_v4/wo_a.py:55-84.
// hc_mix     the hyper-connection low-rank mix of Qwen4-exp at decode sizes: acc = x . W_down^T (FP32),
//            t = BF16(silu(acc / hc)), gate = sigmoid(t . W_up^T) over hc groups of hs columns, and
//            out[m, j] = (1 / hc) * sum_g gate[m, g, j] * x[m, g * hs + j]. Two kernels in stream order (the down
//            projection, then the gated up projection with its epilogue), deterministic: no atomics and no grid
//            barrier. Reference: xtier/packs/qwen4_exp/hc_mix.py:45-116 (same arithmetic; the reference accumulates
//            the down projection with atomics behind a grid barrier).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "params.h"

namespace xt {

// ------------------------------------------------------------------------------------------------------- mhc_post
__global__ void __launch_bounds__(256) mhc_post_kernel(const __nv_bfloat16 *__restrict__ x,
                                                       const __nv_bfloat16 *__restrict__ res,
                                                       const float *__restrict__ post, const float *__restrict__ comb,
                                                       __nv_bfloat16 *__restrict__ out, int M, int H) {
    const int per_row = H / 8;
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    if (i >= (long long)M * per_row) return;
    const int m = int(i / per_row), c = int(i % per_row) * 8;
    float xv[8], rv[4][8];
    auto load8 = [](const __nv_bfloat16 *p, float (&v)[8]) {
        const uint4 w = *reinterpret_cast<const uint4 *>(p);
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(h[k]);
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
        }
    };
    load8(x + size_t(m) * H + c, xv);
#pragma unroll
    for (int j = 0; j < 4; ++j) load8(res + (size_t(m) * 4 + j) * H + c, rv[j]);
#pragma unroll
    for (int o = 0; o < 4; ++o) {
        const float p = post[m * 4 + o];
        const float c0 = comb[m * 16 + 0 * 4 + o], c1 = comb[m * 16 + 1 * 4 + o];
        const float c2 = comb[m * 16 + 2 * 4 + o], c3 = comb[m * 16 + 3 * 4 + o];
        uint4 w;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&w);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float u[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int q = 2 * k + e;
                const float px = __fmul_rn(p, xv[q]);
                const float s0 = __fadd_rn(__fmul_rn(c0, rv[0][q]), __fmul_rn(c1, rv[1][q]));
                const float s1 = __fadd_rn(s0, __fmul_rn(c2, rv[2][q]));
                const float s2 = __fadd_rn(s1, __fmul_rn(c3, rv[3][q]));
                u[e] = __fadd_rn(px, s2);
            }
            h[k] = __floats2bfloat162_rn(u[0], u[1]);
        }
        *reinterpret_cast<uint4 *>(out + (size_t(m) * 4 + o) * H + c) = w;
    }
}

// ---------------------------------------------------------------------------------------------------------- wo_a
constexpr int WA_ROWS = 32, WA_THREADS = 256, WA_TB = 16, WA_HC = 256;

// 8 E4M3 bytes -> 8 floats (hardware conversion, two values per instruction)
XT_DEV void wa_e4m3x8(uint2 w, float (&v)[8]) {
    const uint32_t words[2] = {w.x, w.y};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
                static_cast<__nv_fp8x2_storage_t>((words[q] >> (16 * k)) & 0xFFFF), __NV_E4M3);
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
            v[4 * q + 2 * k] = f.x;
            v[4 * q + 2 * k + 1] = f.y;
        }
    }
}

XT_DEV void wa_bf16x8(uint4 w, float (&v)[8]) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&w);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}

template <bool FP8>
__global__ void __launch_bounds__(WA_THREADS) wo_a_kernel(const __nv_bfloat16 *__restrict__ o, int64_t o_st,
                                                          int64_t o_sg, const uint8_t *__restrict__ w8,
                                                          const __nv_bfloat16 *__restrict__ wb,
                                                          const float *__restrict__ scale, int s_stride,
                                                          __nv_bfloat16 *__restrict__ out, int64_t out_st,
                                                          int64_t out_sg, int T, int R, int D) {
    __shared__ __align__(16) __nv_bfloat16 os[WA_TB][WA_HC];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.y;
    const int r0 = blockIdx.x * WA_ROWS + warp * 4;   // this warp's four weight rows
    for (int tb = 0; tb < T; tb += WA_TB) {
        float acc[4][WA_TB];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
#pragma unroll
            for (int t = 0; t < WA_TB; ++t) acc[rr][t] = 0.f;
        for (int h0 = 0; h0 < D; h0 += WA_HC) {
            __syncthreads();
            for (int q = threadIdx.x; q < WA_TB * WA_HC / 8; q += WA_THREADS) {   // the tokens' activations
                const int t = q / (WA_HC / 8), c = (q % (WA_HC / 8)) * 8;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (tb + t < T && h0 + c < D)
                    v = *reinterpret_cast<const uint4 *>(o + (tb + t) * o_st + g * o_sg + h0 + c);
                *reinterpret_cast<uint4 *>(&os[t][c]) = v;
            }
            __syncthreads();
            const int h = h0 + lane * 8;
            if (h >= D) continue;
            float wv[4][8];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const size_t row = size_t(g) * R + r0 + rr;
                if (FP8) {
                    wa_e4m3x8(*reinterpret_cast<const uint2 *>(w8 + row * D + h), wv[rr]);
                    const float s = scale[(row / 32) * s_stride + h / 32];
#pragma unroll
                    for (int e = 0; e < 8; ++e) wv[rr][e] *= s;
                } else {
                    wa_bf16x8(*reinterpret_cast<const uint4 *>(wb + row * D + h), wv[rr]);
                }
            }
#pragma unroll
            for (int t = 0; t < WA_TB; ++t) {
                float ov[8];
                wa_bf16x8(*reinterpret_cast<const uint4 *>(&os[t][lane * 8]), ov);
#pragma unroll
                for (int rr = 0; rr < 4; ++rr)
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[rr][t] = fmaf(wv[rr][e], ov[e], acc[rr][t]);
            }
        }
        // every lane ends with the 64 totals; lane L writes totals L and L + 32
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
#pragma unroll
            for (int t = 0; t < WA_TB; ++t)
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) acc[rr][t] += __shfl_xor_sync(0xffffffffu, acc[rr][t], off);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int idx = lane + 32 * half, rr = idx / WA_TB, t = idx % WA_TB;
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < 4 * WA_TB; ++q)
                if (q == idx) v = acc[q / WA_TB][q % WA_TB];
            if (tb + t < T) out[(tb + t) * out_st + g * out_sg + r0 + rr] = __float2bfloat16(v);
        }
    }
}

// -------------------------------------------------------------------------------------------------------- hc_mix
constexpr int HM_ROWS = 16, HM_THREADS = 256, HM_KC = 1024;

XT_DEV float hm_sigmoid(float v) { return 1.f / (1.f + __expf(-v)); }

// acc [HM_ROWS, L] FP32 = x [rows, K] . w_down [L, K]^T (rows past `rows` zero): one warp per weight row, x in
// shared memory in 1024-column chunks
__global__ void __launch_bounds__(HM_THREADS) hc_down_kernel(const __nv_bfloat16 *__restrict__ x,
                                                             const __nv_bfloat16 *__restrict__ wd,
                                                             float *__restrict__ acc, int rows, int K, int L) {
    __shared__ __align__(16) __nv_bfloat16 xs[HM_ROWS][HM_KC];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * (HM_THREADS / 32) + warp;
    float a[HM_ROWS];
#pragma unroll
    for (int m = 0; m < HM_ROWS; ++m) a[m] = 0.f;
    for (int k0 = 0; k0 < K; k0 += HM_KC) {
        __syncthreads();
        for (int q = threadIdx.x; q < HM_ROWS * HM_KC / 8; q += HM_THREADS) {
            const int m = q / (HM_KC / 8), c = (q % (HM_KC / 8)) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m < rows && k0 + c < K) v = *reinterpret_cast<const uint4 *>(x + size_t(m) * K + k0 + c);
            *reinterpret_cast<uint4 *>(&xs[m][c]) = v;
        }
        __syncthreads();
        if (n >= L) continue;
        for (int c = lane * 8; c < HM_KC && k0 + c < K; c += 256) {
            float wv[8];
            wa_bf16x8(*reinterpret_cast<const uint4 *>(wd + size_t(n) * K + k0 + c), wv);
#pragma unroll
            for (int m = 0; m < HM_ROWS; ++m) {
                float xv[8];
                wa_bf16x8(*reinterpret_cast<const uint4 *>(&xs[m][c]), xv);
#pragma unroll
                for (int e = 0; e < 8; ++e) a[m] = fmaf(wv[e], xv[e], a[m]);
            }
        }
    }
    if (n >= L) return;
#pragma unroll
    for (int m = 0; m < HM_ROWS; ++m)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a[m] += __shfl_xor_sync(0xffffffffu, a[m], off);
    if (lane < HM_ROWS) {
        float v = 0.f;
#pragma unroll
        for (int m = 0; m < HM_ROWS; ++m)
            if (m == lane) v = a[m];
        acc[size_t(lane) * L + n] = v;
    }
}

// out [rows, hs] = inv_hc * sum_g sigmoid(t . w_up[g * hs + j]) * x[m, g * hs + j] with t = BF16(silu(acc * inv_hc))
// (t in shared memory, computed by every CTA); one warp per output column j
__global__ void __launch_bounds__(HM_THREADS) hc_up_kernel(const float *__restrict__ acc,
                                                           const __nv_bfloat16 *__restrict__ x,
                                                           const __nv_bfloat16 *__restrict__ wu,
                                                           __nv_bfloat16 *__restrict__ out, int rows, int L, int hc,
                                                           int hs, float inv_hc) {
    extern __shared__ __align__(16) uint8_t hm_smem[];
    __nv_bfloat16 *ts = reinterpret_cast<__nv_bfloat16 *>(hm_smem);   // [HM_ROWS][L]
    for (int q = threadIdx.x; q < HM_ROWS * L; q += HM_THREADS) {
        const int m = q / L;
        float v = 0.f;
        if (m < rows) {
            const float a = acc[q] * inv_hc;
            v = a * hm_sigmoid(a);
        }
        ts[q] = __float2bfloat16(v);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * (HM_THREADS / 32) + warp;
    if (j >= hs) return;
    float gsum[HM_ROWS];
#pragma unroll
    for (int m = 0; m < HM_ROWS; ++m) gsum[m] = 0.f;
    for (int g = 0; g < hc; ++g) {
        float d[HM_ROWS];
#pragma unroll
        for (int m = 0; m < HM_ROWS; ++m) d[m] = 0.f;
        const __nv_bfloat16 *wrow = wu + (size_t(g) * hs + j) * L;
        for (int r = lane * 8; r < L; r += 256) {
            float wv[8];
            wa_bf16x8(*reinterpret_cast<const uint4 *>(wrow + r), wv);
#pragma unroll
            for (int m = 0; m < HM_ROWS; ++m) {
                float tv[8];
                wa_bf16x8(*reinterpret_cast<const uint4 *>(ts + m * L + r), tv);
#pragma unroll
                for (int e = 0; e < 8; ++e) d[m] = fmaf(wv[e], tv[e], d[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < HM_ROWS; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) d[m] += __shfl_xor_sync(0xffffffffu, d[m], off);
            if (m < rows) gsum[m] += hm_sigmoid(d[m]) * __bfloat162float(x[size_t(m) * hc * hs + size_t(g) * hs + j]);
        }
    }
    if (lane < rows) {
        float v = 0.f;
#pragma unroll
        for (int m = 0; m < HM_ROWS; ++m)
            if (m == lane) v = gsum[m];
        out[size_t(lane) * hs + j] = __float2bfloat16(v * inv_hc);
    }
}

}  // namespace xt

using namespace xt;

extern "C" {

// x [M, H] BF16, res [M, 4, H] BF16, post [M, 4] FP32, comb [M, 4, 4] FP32 -> out [M, 4, H] BF16 (all contiguous)
int xt_mhc_post(const void *x, const void *res, const float *post, const float *comb, void *out, int M, int H,
                cudaStream_t stream) {
    if (M <= 0) return 0;
    if (H % 8) return -2;
    const long long n = (long long)M * (H / 8);
    mhc_post_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(res), post, comb,
        static_cast<__nv_bfloat16 *>(out), M, H);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// out[t, g, r] = sum_h o[t, g, h] * W[g, r, h]; o and out strided views (element strides; o's 16-byte aligned, unit
// stride along h), W [G, R, D] contiguous: FP8 E4M3 w8 with scale [G * R / 32, D / 32] (row stride s_stride), or BF16
// wb (w8 null). R % 32 == 0, D % 32 == 0.
int xt_wo_a(const void *o, int64_t o_st, int64_t o_sg, const void *w8, const void *wb, const float *scale,
            int s_stride, void *out, int64_t out_st, int64_t out_sg, int T, int G, int R, int D, cudaStream_t stream) {
    if (T <= 0) return 0;
    if (R % WA_ROWS || D % 32 || (o_st | o_sg) % 8 || reinterpret_cast<uintptr_t>(o) % 16 || (!w8 && !wb) ||
        (w8 && !scale))
        return -2;
    dim3 grid(R / WA_ROWS, G);
    if (w8)
        wo_a_kernel<true><<<grid, WA_THREADS, 0, stream>>>(
            static_cast<const __nv_bfloat16 *>(o), o_st, o_sg, static_cast<const uint8_t *>(w8), nullptr, scale,
            s_stride, static_cast<__nv_bfloat16 *>(out), out_st, out_sg, T, R, D);
    else
        wo_a_kernel<false><<<grid, WA_THREADS, 0, stream>>>(
            static_cast<const __nv_bfloat16 *>(o), o_st, o_sg, nullptr, static_cast<const __nv_bfloat16 *>(wb), scale,
            s_stride, static_cast<__nv_bfloat16 *>(out), out_st, out_sg, T, R, D);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// x [rows, hc * hs], w_down [L, hc * hs], w_up [hc * hs, L] (BF16, contiguous) -> out [rows, hs] BF16; acc: FP32
// workspace of 16 x L. Rows in passes of 16; hs, L multiples of 8.
int xt_hc_mix(const void *x, const void *wd, const void *wu, float *acc, void *out, int rows, int hc, int hs, int L,
              cudaStream_t stream) {
    if (rows <= 0) return 0;
    if (hs % 8 || L % 8 || hc <= 0) return -2;
    const size_t smem = size_t(HM_ROWS) * L * 2;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(hc_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 int(smem)) != cudaSuccess)
        return -4;
    const int K = hc * hs;
    for (int m0 = 0; m0 < rows; m0 += HM_ROWS) {
        const int r = rows - m0 < HM_ROWS ? rows - m0 : HM_ROWS;
        const __nv_bfloat16 *xp = static_cast<const __nv_bfloat16 *>(x) + size_t(m0) * K;
        hc_down_kernel<<<(L + 7) / 8, HM_THREADS, 0, stream>>>(xp, static_cast<const __nv_bfloat16 *>(wd), acc, r,
                                                               K, L);
        hc_up_kernel<<<(hs + 7) / 8, HM_THREADS, smem, stream>>>(acc, xp, static_cast<const __nv_bfloat16 *>(wu),
                                                                 static_cast<__nv_bfloat16 *>(out) + size_t(m0) * hs,
                                                                 r, L, hc, hs, 1.f / float(hc));
        if (cudaGetLastError() != cudaSuccess) return -1;
    }
    return 0;
}

}  // extern "C"
