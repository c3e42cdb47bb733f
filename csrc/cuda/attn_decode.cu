// GQA decode attention over a contiguous BF16 KV cache [B, Hkv, L, D=128], split over the keys (flash-decoding).
//
// Grid (splits, Hkv, B), 4 warps. A CTA takes the G = Hq/Hkv query heads of one KV head and a contiguous key range,
// walked in tiles of 128 keys with an online softmax:
//   scores  each warp takes 32 keys, one per lane: the lane loads its key's 256-byte row (16 independent 16-byte
//           loads in flight) and forms the G head dots against the pre-scaled queries in shared memory (broadcast
//           reads), so no cross-lane reduction is needed.
//   softmax one warp per head: tile max, running max and sum, exp2 in place.
//   values  lane l accumulates dims 4l..4l+3 of all G heads; the probabilities are read from shared memory as
//           [key][head] so G heads of one key are one or two vector loads.
// Each split writes its unnormalized output, max and sum to a workspace; the last CTA of a (batch, KV head) to finish
// merges the splits (an arrival counter that it resets), so one launch does the whole step and the grid shape does not
// depend on the sequence length (graph capture). Sequence lengths are read from device memory.
// Reference parity: the reference leaves dense decode attention to SGLang's backends; this kernel is the dense
// attention of the Qwen3-style config (GQA 32/4, head dim 128).
#include "common.cuh"
#include "params.h"

namespace xt {

constexpr int AD_WARPS = 4;
constexpr int AD_TILE = 32 * AD_WARPS;
constexpr int AD_D = 128;


template <int G>
__global__ void __launch_bounds__(AD_WARPS * 32) attn_decode_kernel(AttnDecodeParams p) {
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int N = p.seqlens[b];
    int chunk = (N + p.splits - 1) / p.splits;
    chunk = (chunk + 31) & ~31;
    const int k_begin = split * chunk, k_end = min(N, k_begin + chunk);

    // the score tile and the final cross-warp reduction never live at the same time: one buffer holds either
    __shared__ __align__(16) float buf[AD_WARPS * G * AD_D];
    float(&S)[AD_TILE][G] = *reinterpret_cast<float(*)[AD_TILE][G]>(buf);
    float(&red)[AD_WARPS][G][AD_D] = *reinterpret_cast<float(*)[AD_WARPS][G][AD_D]>(buf);
    __shared__ __align__(16) float qs[G][AD_D];
    __shared__ float m_run[G], l_run[G], alpha[G];

    const __nv_bfloat16 *qb = p.q + (size_t(b) * p.Hq + size_t(kvh) * G) * AD_D;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) qs[i / AD_D][i % AD_D] = __bfloat162float(qb[i]) * p.scale_log2;
    if (threadIdx.x < G) {
        m_run[threadIdx.x] = -INFINITY;
        l_run[threadIdx.x] = 0.f;
    }
    __syncthreads();
    float acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;

    const size_t head_off = (size_t(b) * p.Hkv + kvh) * p.L;
    const __nv_bfloat16 *K = p.kc + head_off * AD_D;
    const __nv_bfloat16 *V = p.vc + head_off * AD_D;

    for (int t0 = k_begin; t0 < k_end; t0 += AD_TILE) {
        // ---- scores: lane = key
        {
            const int key = t0 + warp * 32 + lane;
            const bool valid = key < k_end;
            const uint4 *kr = reinterpret_cast<const uint4 *>(K + size_t(valid ? key : k_begin) * AD_D);
            uint4 kv[AD_D / 8];
#pragma unroll
            for (int c = 0; c < AD_D / 8; ++c) kv[c] = kr[c];
            float s[G];
#pragma unroll
            for (int h = 0; h < G; ++h) s[h] = 0.f;
#pragma unroll
            for (int c = 0; c < AD_D / 8; ++c) {
                const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&kv[c]);
                float kf[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 f = __bfloat1622float2(k2[i]);
                    kf[2 * i] = f.x;
                    kf[2 * i + 1] = f.y;
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(&qs[h][c * 8]);
                    const float4 q1 = *reinterpret_cast<const float4 *>(&qs[h][c * 8 + 4]);
                    s[h] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                            q1.z * kf[6] + q1.w * kf[7];
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) S[warp * 32 + lane][h] = valid ? s[h] : -INFINITY;
        }
        __syncthreads();
        // ---- online softmax per head
        for (int h = warp; h < G; h += AD_WARPS) {
            float mx = -INFINITY;
            for (int i = lane; i < AD_TILE; i += 32) mx = fmaxf(mx, S[i][h]);
            mx = warp_max(mx);
            const float m_old = m_run[h];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int i = lane; i < AD_TILE; i += 32) {
                float e = (m_new == -INFINITY) ? 0.f : exp2f(S[i][h] - m_new);
                S[i][h] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float a = (m_old == -INFINITY) ? 0.f : exp2f(m_old - m_new);
                alpha[h] = a;
                l_run[h] = l_run[h] * a + sum;
                m_run[h] = m_new;
            }
        }
        __syncthreads();
        // ---- values: lane owns dims 4l..4l+3, the warp walks its 32 keys eight at a time
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float a = alpha[h];
#pragma unroll
            for (int d = 0; d < 4; ++d) acc[h][d] *= a;
        }
        const int nk = min(32, k_end - (t0 + warp * 32));
        for (int i0 = 0; i0 < nk; i0 += 8) {
            uint2 vv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int key = t0 + warp * 32 + min(i0 + i, nk - 1);
                vv[i] = *reinterpret_cast<const uint2 *>(V + size_t(key) * AD_D + lane * 4);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i0 + i >= nk) break;
                const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&vv[i]);
                float2 f0 = __bfloat1622float2(u2[0]), f1 = __bfloat1622float2(u2[1]);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float pr = S[warp * 32 + i0 + i][h];
                    acc[h][0] += pr * f0.x;
                    acc[h][1] += pr * f0.y;
                    acc[h][2] += pr * f1.x;
                    acc[h][3] += pr * f1.y;
                }
            }
        }
        __syncthreads();
    }
    // ---- combine the warps, write this split's partial
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d) red[warp][h][lane * 4 + d] = acc[h][d];
    __syncthreads();
    const size_t part = ((size_t(b) * p.Hkv + kvh) * p.splits + split) * G;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) {
        const int h = i / AD_D, d = i % AD_D;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < AD_WARPS; ++w) s += red[w][h][d];
        p.ws_o[part * AD_D + i] = s;
    }
    if (threadIdx.x < G) {
        p.ws_ml[(part + threadIdx.x) * 2] = m_run[threadIdx.x];
        p.ws_ml[(part + threadIdx.x) * 2 + 1] = l_run[threadIdx.x];
    }
    // ---- the last split to arrive merges
    __shared__ bool last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned prev = atomicAdd(&p.counters[b * p.Hkv + kvh], 1u);
        last = prev == unsigned(p.splits) - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // merge: every split's (max, sum) into shared memory at once, one weight per (split, head), then each output
    // element is a weighted sum over the splits whose loads are all independent (no serial L2 round trips)
    constexpr int MAX_SPLITS = 64;
    __shared__ float wsplit[MAX_SPLITS][G];
    const size_t base = (size_t(b) * p.Hkv + kvh) * p.splits * G;
    float *mls = buf;   // the score / reduction buffer is free again
    for (int i = threadIdx.x; i < p.splits * G * 2; i += blockDim.x) mls[i] = __ldcg(p.ws_ml + base * 2 + i);
    __syncthreads();
    if (threadIdx.x < G) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int s = 0; s < p.splits; ++s) M = fmaxf(M, mls[(s * G + h) * 2]);
        float L = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float ms = mls[(s * G + h) * 2];
            const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
            wsplit[s][h] = f;
            L += mls[(s * G + h) * 2 + 1] * f;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int s = 0; s < p.splits; ++s) wsplit[s][h] *= inv;
    }
    __syncthreads();
    // four consecutive dims per thread (16-byte loads), all splits' loads of a group issued back to back
    for (int i = threadIdx.x * 4; i < G * AD_D; i += blockDim.x * 4) {
        const int h = i / AD_D;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 *src = reinterpret_cast<const float4 *>(p.ws_o + base * AD_D + i);
        const size_t stride4 = size_t(G) * AD_D / 4;   // float4s between consecutive splits
        int s = 0;
        for (; s + 8 <= p.splits; s += 8) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + (s + j) * stride4);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float wgt = wsplit[s + j][h];
                O.x += v[j].x * wgt;
                O.y += v[j].y * wgt;
                O.z += v[j].z * wgt;
                O.w += v[j].w * wgt;
            }
        }
        for (; s < p.splits; ++s) {
            const float4 v = __ldcg(src + s * stride4);
            const float wgt = wsplit[s][h];
            O.x += v.x * wgt;
            O.y += v.y * wgt;
            O.z += v.z * wgt;
            O.w += v.w * wgt;
        }
        __nv_bfloat16 *dst = p.out + (size_t(b) * p.Hq + size_t(kvh) * G + h) * AD_D + i % AD_D;
        reinterpret_cast<__nv_bfloat162 *>(dst)[0] = __floats2bfloat162_rn(O.x, O.y);
        reinterpret_cast<__nv_bfloat162 *>(dst)[1] = __floats2bfloat162_rn(O.z, O.w);
    }
    if (threadIdx.x == 0) p.counters[b * p.Hkv + kvh] = 0;
}

}  // namespace xt

using namespace xt;

extern "C" int xt_attn_decode(const AttnDecodeParams *pp, int B, cudaStream_t stream) {
    AttnDecodeParams p = *pp;
    const int G = p.Hq / p.Hkv;
    if (p.Hq % p.Hkv || p.splits < 1 || p.splits > 64) return -2;
    dim3 grid(p.splits, p.Hkv, B);
    switch (G) {
        case 1: attn_decode_kernel<1><<<grid, AD_WARPS * 32, 0, stream>>>(p); break;
        case 2: attn_decode_kernel<2><<<grid, AD_WARPS * 32, 0, stream>>>(p); break;
        case 4: attn_decode_kernel<4><<<grid, AD_WARPS * 32, 0, stream>>>(p); break;
        case 8: attn_decode_kernel<8><<<grid, AD_WARPS * 32, 0, stream>>>(p); break;
        case 16: attn_decode_kernel<16><<<grid, AD_WARPS * 32, 0, stream>>>(p); break;
        default: return -3;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
