// Normalization and rotary kernels of the dense path (BF16 in and out, FP32 arithmetic).
//
//   add_rmsnorm       residual += x (rounded to BF16, as the model's residual stream is BF16), out = RMSNorm(residual)
//                     * w; without a residual it is a plain RMSNorm. One CTA per token, 16-byte accesses.
//   qk_norm_rope_kv   splits a fused QKV row into heads, applies the optional per-head RMSNorm of Q and K (Qwen3),
//                     NeoX-style RoPE (rotate half) at the token's position, writes Q and appends K, V to the cache
//                     [B, Hkv, L, D] at (cache_batch[t], positions[t]). One warp per (token, head); each lane owns
//                     dims {2l, 2l+1} and their rotation partners {2l+D/2, 2l+1+D/2}, so the rotation is lane-local.
#include "common.cuh"
#include "params.h"

namespace xt {

constexpr int NORM_THREADS = 256;

__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(const __nv_bfloat16 *x, __nv_bfloat16 *residual,
                                                                   const __nv_bfloat16 *w, __nv_bfloat16 *out, int H,
                                                                   float eps) {
    const int t = blockIdx.x;
    const __nv_bfloat16 *xr = x + size_t(t) * H;
    __nv_bfloat16 *rr = residual ? residual + size_t(t) * H : nullptr;
    __shared__ float red[NORM_THREADS / 32];
    pdl_wait();
    pdl_trigger();
    float ss = 0.f;
    // pass 1: sum (and store the new residual)
    for (int i = threadIdx.x * 8; i < H; i += NORM_THREADS * 8) {
        uint4 a = *reinterpret_cast<const uint4 *>(xr + i);
        __nv_bfloat162 *a2 = reinterpret_cast<__nv_bfloat162 *>(&a);
        if (rr) {
            uint4 b = *reinterpret_cast<const uint4 *>(rr + i);
            const __nv_bfloat162 *b2 = reinterpret_cast<const __nv_bfloat162 *>(&b);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 fa = __bfloat1622float2(a2[j]), fb = __bfloat1622float2(b2[j]);
                a2[j] = __floats2bfloat162_rn(fa.x + fb.x, fa.y + fb.y);
            }
            *reinterpret_cast<uint4 *>(rr + i) = a;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 f = __bfloat1622float2(a2[j]);
            ss += f.x * f.x + f.y * f.y;
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < NORM_THREADS / 32 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = rsqrtf(v / H + eps);
    }
    __syncthreads();
    const float inv = red[0];
    const __nv_bfloat16 *src = rr ? rr : xr;
    for (int i = threadIdx.x * 8; i < H; i += NORM_THREADS * 8) {
        uint4 a = *reinterpret_cast<const uint4 *>(src + i);
        uint4 g = *reinterpret_cast<const uint4 *>(w + i);
        __nv_bfloat162 *a2 = reinterpret_cast<__nv_bfloat162 *>(&a);
        const __nv_bfloat162 *g2 = reinterpret_cast<const __nv_bfloat162 *>(&g);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float2 fa = __bfloat1622float2(a2[j]), fg = __bfloat1622float2(g2[j]);
            a2[j] = __floats2bfloat162_rn(fa.x * inv * fg.x, fa.y * inv * fg.y);
        }
        *reinterpret_cast<uint4 *>(out + size_t(t) * H + i) = a;
    }
}


// D == 128: lane l owns dims 2l, 2l+1 (first half) and 64+2l, 65+2l (second half)
__global__ void qk_norm_rope_kv_kernel(RopeParams p) {
    pdl_wait();
    pdl_trigger();
    const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int heads = p.Hq + 2 * p.Hkv;
    const int t = warp_global / heads, h = warp_global % heads;
    if (t >= p.T) return;
    const int D = 128, half = 64;
    const __nv_bfloat16 *src = p.qkv + size_t(t) * heads * D + size_t(h) * D;
    float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(src + 2 * lane));
    float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(src + half + 2 * lane));
    const bool is_q = h < p.Hq, is_k = !is_q && h < p.Hq + p.Hkv;
    const __nv_bfloat16 *nw = is_q ? p.qn : (is_k ? p.kn : nullptr);
    if (nw) {   // the model rounds the normalized head to BF16 before RoPE
        float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
        float inv = rsqrtf(ss / D + p.eps);
        float2 wa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(nw + 2 * lane));
        float2 wb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(nw + half + 2 * lane));
        a.x = __bfloat162float(__float2bfloat16(a.x * inv * wa.x));
        a.y = __bfloat162float(__float2bfloat16(a.y * inv * wa.y));
        b.x = __bfloat162float(__float2bfloat16(b.x * inv * wb.x));
        b.y = __bfloat162float(__float2bfloat16(b.y * inv * wb.y));
    }
    if (is_q || is_k) {
        const float pos = float(p.pos[t]);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = 2 * lane + j;   // frequency index
            const float inv_freq = powf(p.theta, -2.f * i / D);
            float sn, cs;
            sincosf(pos * inv_freq, &sn, &cs);
            float &x1 = j ? a.y : a.x;
            float &x2 = j ? b.y : b.x;
            const float r1 = x1 * cs - x2 * sn, r2 = x2 * cs + x1 * sn;
            x1 = r1;
            x2 = r2;
        }
    }
    __nv_bfloat16 *dst;
    if (is_q) {
        dst = p.q + (size_t(t) * p.Hq + h) * D;
    } else {
        const int kvh = is_k ? h - p.Hq : h - p.Hq - p.Hkv;
        __nv_bfloat16 *cache = is_k ? p.kc : p.vc;
        dst = cache + ((size_t(p.batch[t]) * p.Hkv + kvh) * p.L + (p.slot ? p.slot[t] : p.pos[t])) * D;
    }
    *reinterpret_cast<__nv_bfloat162 *>(dst + 2 * lane) = __floats2bfloat162_rn(a.x, a.y);
    *reinterpret_cast<__nv_bfloat162 *>(dst + half + 2 * lane) = __floats2bfloat162_rn(b.x, b.y);
}

}  // namespace xt

using namespace xt;

extern "C" {

int xt_add_rmsnorm(const void *x, void *residual, const void *w, void *out, int T, int H, float eps,
                   cudaStream_t stream) {
    if (H % 8) return -2;
    const cudaError_t e = xt_launch(add_rmsnorm_kernel, dim3(T), dim3(NORM_THREADS), 0, stream,
                                    static_cast<const __nv_bfloat16 *>(x), static_cast<__nv_bfloat16 *>(residual),
                                    static_cast<const __nv_bfloat16 *>(w), static_cast<__nv_bfloat16 *>(out), H, eps);
    return e == cudaSuccess ? 0 : -1;
}

int xt_qk_norm_rope_kv(const RopeParams *p, cudaStream_t stream) {
    if (p->D != 128) return -2;
    const int warps = p->T * (p->Hq + 2 * p->Hkv);
    const int threads = 256;
    const cudaError_t e = xt_launch(qk_norm_rope_kv_kernel, dim3((warps * 32 + threads - 1) / threads),
                                    dim3(threads), 0, stream, *p);
    return e == cudaSuccess ? 0 : -1;
}

}  // extern "C"
