// The MLA decode step's small operations around the attention kernel (sm_100a). At decode sizes (a few to a few
// dozen tokens per GPU) each is a stream of a few MB of weights or a per-token vector operation, so these are
// CUDA-core kernels built to keep loads in flight, and each replaces a chain of framework ops:
//
//   mla_prep     one CTA per token: the fused [q_a | kv_a] projection row (q_lora + kv_lora + rope values) ->
//                RMSNorm of the query's low-rank part (BF16 out, the q_b projection's input); RMSNorm of the compressed
//                KV, rounded to BF16 and written into the NVFP4 latent cache at the token's slot (E2M1 codes and one
//                E4M3 scale per 16 values, the encoding of mla_kv_write); NeoX RoPE of the rotary key at the token's
//                position, BF16 into the cache; and optionally the BF16 latent row itself.
//   silu_mul     the dense MLP's activation: [T, 2I] (gate rows then up rows of the fused projection) ->
//                SiLU(gate) * up in FP32, BF16 out [T, I].
//   head_gemm    per head: Y[t, h, :N] = X[t, h, :K] . W[h] (W[h] is [K, N] row-major), grid (heads, N / 64), K split
//                over the warps; the query absorption (q_nope . W_uk, K 128 -> N 512, with the query's rotary dims rotated by an extra
//                column block of CTAs) and the value un-absorption (o_latent . W_uv^T, K 512 -> N 128).
//
// Reference parity: the reference runs these steps inside SGLang's DeepSeek model code (FlashMLA decode with the
// absorbed query); xtier/packs/deepseek_v4/sparse_mla.py:1-20 describes the quantized-KV sparse MLA they feed.
#include "common.cuh"
#include "params.h"

#include <algorithm>

namespace xt {

constexpr int MP_THREADS = 256;
constexpr int HG_COLS = 64;      // output columns per CTA
constexpr int HG_TOK = 16;       // tokens per pass (registers and shared-memory chunk)

// NeoX rotation of the pair (a, b) = (x[i], x[i + d/2]) at position pos, frequency index i of d rotary dims
XT_DEV float2 rope_pair(float a, float b, float pos, int i, int d, float theta) {
    const float inv_freq = powf(theta, -2.f * float(i) / float(d));
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    return make_float2(a * cs - b * sn, b * cs + a * sn);
}

XT_DEV float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < MP_THREADS / 32; ++w) s += red[w];
    return s;
}

// in [T, ld]: q_lora values, then kv_lora latent values, then rope values (ld >= q_lora + kv_lora + 64)
__global__ void __launch_bounds__(MP_THREADS) mla_prep_kernel(const __nv_bfloat16 *__restrict__ in, int ld,
                                                              int q_lora, const __nv_bfloat16 *__restrict__ q_norm,
                                                              const __nv_bfloat16 *__restrict__ kv_norm,
                                                              const int32_t *__restrict__ pos,
                                                              const int64_t *__restrict__ slot, float eps,
                                                              float theta, __nv_bfloat16 *__restrict__ q_out,
                                                              uint8_t *codes, uint8_t *scales, __nv_bfloat16 *rope,
                                                              __nv_bfloat16 *lat_out) {
    constexpr int L = 512, R = 64;
    __shared__ float red[MP_THREADS / 32];
    __shared__ float lat[L];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, tid = threadIdx.x;
    const __nv_bfloat16 *row = in + size_t(t) * ld;
    // query low-rank part: RMSNorm (the model's ops.rmsnorm: FP32 sum of squares, BF16 out)
    float ss = 0.f;
    for (int i = tid; i < q_lora; i += MP_THREADS) {
        const float v = bf16_to_f(row[i]);
        ss += v * v;
    }
    const float qinv = rsqrtf(block_sum(ss, red) / float(q_lora) + eps);
    for (int i = tid; i < q_lora; i += MP_THREADS)
        q_out[size_t(t) * q_lora + i] = __float2bfloat16(bf16_to_f(row[i]) * qinv * bf16_to_f(q_norm[i]));
    // compressed KV: RMSNorm, rounded to BF16 (the cache's input values)
    const __nv_bfloat16 *c = row + q_lora;
    ss = 0.f;
    for (int i = tid; i < L; i += MP_THREADS) {
        const float v = bf16_to_f(c[i]);
        ss += v * v;
    }
    const float cinv = rsqrtf(block_sum(ss, red) / float(L) + eps);
    for (int i = tid; i < L; i += MP_THREADS)
        lat[i] = bf16_to_f(__float2bfloat16(bf16_to_f(c[i]) * cinv * bf16_to_f(kv_norm[i])));
    __syncthreads();
    const size_t s = size_t(slot[t]);
    const int warp = tid >> 5, lane = tid & 31;
    if (warp == 0) {   // lane = one block of 16 latent values -> 8 code bytes + one E4M3 scale
        const float *v = lat + lane * 16;
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const uint8_t sc = f32_to_e4m3(amax / 6.f);
        const float sf = e4m3_to_f(sc);
        const float inv = sf > 0.f ? 1.f / sf : 0.f;
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t acc = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                acc |= uint32_t(f32x2_to_e2m1(v[h * 8 + 2 * i] * inv, v[h * 8 + 2 * i + 1] * inv)) << (8 * i);
            w[h] = acc;
        }
        *reinterpret_cast<uint2 *>(codes + s * (L / 2) + lane * 8) = make_uint2(w[0], w[1]);
        scales[s * (L / 16) + lane] = sc;
    } else if (warp == 1) {   // rotary key: lane i rotates the pair (i, i + 32)
        const __nv_bfloat16 *kr = c + L;
        const float2 r = rope_pair(bf16_to_f(kr[lane]), bf16_to_f(kr[lane + R / 2]), float(pos[t]), lane, R, theta);
        const __nv_bfloat16 a = __float2bfloat16(r.x), b = __float2bfloat16(r.y);
        rope[s * R + lane] = a;
        rope[s * R + lane + R / 2] = b;
        if (lat_out) {
            lat_out[size_t(t) * (L + R) + L + lane] = a;
            lat_out[size_t(t) * (L + R) + L + lane + R / 2] = b;
        }
    }
    if (lat_out)
        for (int i = tid; i < L; i += MP_THREADS) lat_out[size_t(t) * (L + R) + i] = __float2bfloat16(lat[i]);
}

// grid (heads, N / 64 [+ 1 rotary block]). The 8 warps split K; lane c owns columns n0 + 2c, n0 + 2c + 1 and keeps
// the sums of up to HG_TOK tokens in registers, so every weight is loaded once per CTA (eight loads in flight per lane);
// the warps' partial sums meet in shared memory and are added in warp order.
__global__ void __launch_bounds__(MP_THREADS) head_gemm_kernel(HeadGemmParams p) {
    extern __shared__ __align__(16) uint8_t hg_smem[];
    constexpr int NW = MP_THREADS / 32;
    __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(hg_smem);                        // [HG_TOK][K]
    float *red = reinterpret_cast<float *>(hg_smem + size_t(HG_TOK) * p.K * 2);           // [NW][HG_TOK][64]
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, c = tid & 31;
    const int nblk = p.N / HG_COLS;
    pdl_wait();
    pdl_trigger();
    if (int(blockIdx.y) == nblk) {   // the rotary dims of every token of this head
        const int half = p.rope_dims / 2;
        for (int i = tid; i < p.T * half; i += MP_THREADS) {
            const int t = i / half, j = i % half;
            const __nv_bfloat16 *xr = p.x + t * p.xs_t + h * p.xs_h + p.rope_x;
            const float2 r = rope_pair(bf16_to_f(xr[j]), bf16_to_f(xr[j + half]), float(p.pos[t]), j, p.rope_dims,
                                       p.theta);
            __nv_bfloat16 *yr = p.y + t * p.ys_t + h * p.ys_h + p.rope_y;
            yr[j] = __float2bfloat16(r.x);
            yr[j + half] = __float2bfloat16(r.y);
        }
        return;
    }
    const int n0 = blockIdx.y * HG_COLS;
    const int kw = p.K / NW;                 // this warp's K slice (K % 64 == 0)
    const int k0w = warp * kw;
    const __nv_bfloat16 *W = p.w + size_t(h) * p.K * p.N + n0 + 2 * c;
    for (int t0 = 0; t0 < p.T; t0 += HG_TOK) {
        const int nt = min(HG_TOK, p.T - t0);
        __syncthreads();
        for (int i = tid; i < nt * (p.K / 8); i += MP_THREADS) {
            const int t = i / (p.K / 8), kc = i % (p.K / 8);
            reinterpret_cast<uint4 *>(xs + size_t(t) * p.K)[kc] =
                *reinterpret_cast<const uint4 *>(p.x + (t0 + t) * p.xs_t + h * p.xs_h + kc * 8);
        }
        __syncthreads();
        float acc[HG_TOK][2];
#pragma unroll
        for (int t = 0; t < HG_TOK; ++t) acc[t][0] = acc[t][1] = 0.f;
        for (int k0 = k0w; k0 < k0w + kw; k0 += 8) {
            float2 wf[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                wf[u] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(W + size_t(k0 + u) * p.N));
#pragma unroll
            for (int t = 0; t < HG_TOK; ++t) {
                if (t >= nt) break;
                const uint4 xv = *reinterpret_cast<const uint4 *>(xs + size_t(t) * p.K + k0);
                const __nv_bfloat162 *x2 = reinterpret_cast<const __nv_bfloat162 *>(&xv);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 xf = __bfloat1622float2(x2[u]);
                    acc[t][0] = fmaf(xf.x, wf[2 * u].x, fmaf(xf.y, wf[2 * u + 1].x, acc[t][0]));
                    acc[t][1] = fmaf(xf.x, wf[2 * u].y, fmaf(xf.y, wf[2 * u + 1].y, acc[t][1]));
                }
            }
        }
#pragma unroll
        for (int t = 0; t < HG_TOK; ++t) {
            if (t >= nt) break;
            *reinterpret_cast<float2 *>(red + (size_t(warp) * HG_TOK + t) * HG_COLS + 2 * c) =
                make_float2(acc[t][0], acc[t][1]);
        }
        __syncthreads();
        for (int i = tid; i < nt * 32; i += MP_THREADS) {   // (token, column pair): the warps' sums in warp order
            const int t = i / 32, cc = i % 32;
            float2 s = make_float2(0.f, 0.f);
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float2 v = *reinterpret_cast<const float2 *>(red + (size_t(w) * HG_TOK + t) * HG_COLS + 2 * cc);
                s.x += v.x;
                s.y += v.y;
            }
            *reinterpret_cast<__nv_bfloat162 *>(p.y + (t0 + t) * p.ys_t + h * p.ys_h + n0 + 2 * cc) =
                __floats2bfloat162_rn(s.x, s.y);
        }
    }
}

// in [T, 2I], out [T, I]; two columns per thread
__global__ void __launch_bounds__(MP_THREADS) silu_mul_kernel(const __nv_bfloat16 *__restrict__ in,
                                                              __nv_bfloat16 *__restrict__ out, int T, int I) {
    pdl_wait();
    pdl_trigger();
    const int half = I / 2;
    for (long long i = blockIdx.x * (long long)MP_THREADS + threadIdx.x; i < (long long)T * half;
         i += (long long)gridDim.x * MP_THREADS) {
        const long long t = i / half;
        const int j = int(i % half) * 2;
        const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(in + t * 2 * I + j));
        const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(in + t * 2 * I + I + j));
        const float a = g.x / (1.f + expf(-g.x)) * u.x, b = g.y / (1.f + expf(-g.y)) * u.y;
        *reinterpret_cast<__nv_bfloat162 *>(out + t * I + j) = __floats2bfloat162_rn(a, b);
    }
}

}  // namespace xt

using namespace xt;

// y[t, h, :d] = NeoX RoPE of x[t, h, :d] at pos[t] (strided over tokens and heads); one warp per (token, head)
__global__ void __launch_bounds__(256) rope_heads_kernel(const __nv_bfloat16 *__restrict__ x, int64_t xs_t, int64_t xs_h,
                                                        const int32_t *__restrict__ pos, float theta,
                                                        __nv_bfloat16 *__restrict__ y, int64_t ys_t, int64_t ys_h,
                                                        int T, int H, int d) {
    const long long w = blockIdx.x * 8ll + (threadIdx.x >> 5);
    if (w >= (long long)T * H) return;
    const int t = int(w / H), h = int(w % H), lane = threadIdx.x & 31;
    const __nv_bfloat16 *xr = x + t * xs_t + h * xs_h;
    __nv_bfloat16 *yr = y + t * ys_t + h * ys_h;
    const int half = d / 2;
    for (int i = lane; i < half; i += 32) {
        const float2 r = rope_pair(bf16_to_f(xr[i]), bf16_to_f(xr[i + half]), float(pos[t]), i, d, theta);
        yr[i] = __float2bfloat16(r.x);
        yr[i + half] = __float2bfloat16(r.y);
    }
}

extern "C" {

int xt_mla_prep(const void *in, int ld, int q_lora, const void *q_norm, const void *kv_norm, const int32_t *pos,
                const int64_t *slot, float eps, float theta, void *q_out, void *codes, void *scales, void *rope,
                void *lat_out, int T, cudaStream_t stream) {
    if (T <= 0) return 0;
    if (ld < q_lora + 512 + 64) return -2;
    const cudaError_t e = xt_launch(mla_prep_kernel, dim3(T), dim3(MP_THREADS), 0, stream,
                                    static_cast<const __nv_bfloat16 *>(in), ld, q_lora,
                                    static_cast<const __nv_bfloat16 *>(q_norm),
                                    static_cast<const __nv_bfloat16 *>(kv_norm), pos, slot, eps, theta,
                                    static_cast<__nv_bfloat16 *>(q_out), static_cast<uint8_t *>(codes),
                                    static_cast<uint8_t *>(scales), static_cast<__nv_bfloat16 *>(rope),
                                    static_cast<__nv_bfloat16 *>(lat_out));
    return e == cudaSuccess ? 0 : -1;
}

int xt_silu_mul(const void *in, void *out, int T, int I, cudaStream_t stream) {
    if (T <= 0) return 0;
    if (I % 2) return -2;
    const long long pairs = (long long)T * (I / 2);
    const int grid = int(std::min<long long>((pairs + MP_THREADS - 1) / MP_THREADS, 148 * 16));
    const cudaError_t e = xt_launch(silu_mul_kernel, dim3(grid), dim3(MP_THREADS), 0, stream,
                                    static_cast<const __nv_bfloat16 *>(in), static_cast<__nv_bfloat16 *>(out), T, I);
    return e == cudaSuccess ? 0 : -1;
}

int xt_rope_heads(const void *x, int64_t xs_t, int64_t xs_h, const int32_t *pos, float theta, void *y, int64_t ys_t,
                  int64_t ys_h, int T, int H, int d, cudaStream_t stream) {
    if (T <= 0 || H <= 0) return 0;
    if (d <= 0 || d % 2) return -2;
    const long long warps = (long long)T * H;
    rope_heads_kernel<<<unsigned((warps + 7) / 8), 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(x), xs_t, xs_h,
                                                                     pos, theta, static_cast<__nv_bfloat16 *>(y), ys_t,
                                                                     ys_h, T, H, d);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_head_gemm(const HeadGemmParams *pp, int heads, cudaStream_t stream) {
    const HeadGemmParams &p = *pp;
    if (p.T <= 0) return 0;
    if (p.N % HG_COLS || p.K % 64 || p.K > 1024 || p.xs_t % 8 || p.xs_h % 8 || p.ys_h % 2 || p.ys_t % 2) return -2;
    if (p.rope_dims && (!p.pos || p.rope_dims % 2)) return -2;
    const int smem = HG_TOK * p.K * 2 + (MP_THREADS / 32) * HG_TOK * HG_COLS * 4;
    if (xt_smem_optin(head_gemm_kernel, smem) != cudaSuccess) return -4;
    dim3 grid(heads, p.N / HG_COLS + (p.rope_dims ? 1 : 0));
    const cudaError_t e = xt_launch(head_gemm_kernel, grid, dim3(MP_THREADS), size_t(smem), stream, p);
    return e == cudaSuccess ? 0 : -1;
}

}  // extern "C"
