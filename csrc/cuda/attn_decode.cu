// GQA decode attention over a contiguous BF16 KV cache [B, Hkv, L, D=128], split over the keys (flash-decoding).
//
// Grid (splits, Hkv, B), 4 warps. A CTA takes the G = Hq/Hkv query heads of one KV head and a contiguous key range,
// walked in tiles of 128 keys with an online softmax:
//   scores  each warp takes 32 keys; per key every lane loads 4 dims of K (8 bytes, the warp reads the 256-byte row
//           once), forms G partial dots, and a butterfly reduce-scatter over the lanes (log2(32) + log2(G) shuffles
//           instead of 5 G) leaves each head's full dot on a group of lanes, which writes it to shared memory.
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


// reduce-scatter of G per-lane values: afterwards every lane holds the full (32-lane) sum of value index
// head_of(lane), where head_of(lane) takes log2(G) lane bits from the top (bit 4 first)
template <int G>
XT_DEV float butterfly(float (&v)[G], int lane) {
    int cnt = G;
    int o = 16;
#pragma unroll
    for (int step = 0; (1 << step) < G; ++step) {
        const int half = cnt / 2;
        const bool upper = lane & o;
#pragma unroll
        for (int i = 0; i < G / 2; ++i) {
            if (i < half) {
                float send = upper ? v[i] : v[i + half];
                float keep = upper ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        cnt = half;
        o >>= 1;
    }
    float r = v[0];
    for (; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

template <int G>
XT_DEV int head_of(int lane) {
    int h = 0, o = 16;
    for (int g = G; g > 1; g >>= 1, o >>= 1) h = h * 2 + ((lane & o) ? 1 : 0);
    return h;
}

template <int G>
__global__ void __launch_bounds__(AD_WARPS * 32) attn_decode_kernel(AttnDecodeParams p) {
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int N = p.seqlens[b];
    int chunk = (N + p.splits - 1) / p.splits;
    chunk = (chunk + 31) & ~31;
    const int k_begin = split * chunk, k_end = min(N, k_begin + chunk);

    __shared__ float S[AD_TILE][G];
    __shared__ float m_run[G], l_run[G], alpha[G];
    __shared__ float red[AD_WARPS][G][AD_D];

    // this lane's 4 dims of every head's query, pre-scaled
    float qr[G][4];
    const __nv_bfloat16 *qb = p.q + (size_t(b) * p.Hq + size_t(kvh) * G) * AD_D;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        uint2 u = *reinterpret_cast<const uint2 *>(qb + h * AD_D + lane * 4);
        const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u);
        float2 f0 = __bfloat1622float2(u2[0]), f1 = __bfloat1622float2(u2[1]);
        qr[h][0] = f0.x * p.scale_log2;
        qr[h][1] = f0.y * p.scale_log2;
        qr[h][2] = f1.x * p.scale_log2;
        qr[h][3] = f1.y * p.scale_log2;
    }
    if (threadIdx.x < G) {
        m_run[threadIdx.x] = -INFINITY;
        l_run[threadIdx.x] = 0.f;
    }
    float acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;

    const size_t head_off = (size_t(b) * p.Hkv + kvh) * p.L;
    const __nv_bfloat16 *K = p.kc + head_off * AD_D;
    const __nv_bfloat16 *V = p.vc + head_off * AD_D;
    const int my_head = head_of<G>(lane);
    constexpr int LANES_PER_HEAD = 32 / G;

    for (int t0 = k_begin; t0 < k_end; t0 += AD_TILE) {
        // ---- scores of this warp's 32 keys
#pragma unroll 4
        for (int i = 0; i < 32; ++i) {
            const int key = t0 + warp * 32 + i;
            float v[G];
            if (key < k_end) {
                uint2 u = *reinterpret_cast<const uint2 *>(K + size_t(key) * AD_D + lane * 4);
                const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u);
                float2 f0 = __bfloat1622float2(u2[0]), f1 = __bfloat1622float2(u2[1]);
#pragma unroll
                for (int h = 0; h < G; ++h) v[h] = qr[h][0] * f0.x + qr[h][1] * f0.y + qr[h][2] * f1.x + qr[h][3] * f1.y;
            } else {
#pragma unroll
                for (int h = 0; h < G; ++h) v[h] = 0.f;
            }
            float s = butterfly<G>(v, lane);
            if ((lane % LANES_PER_HEAD) == 0) S[warp * 32 + i][my_head] = key < k_end ? s : -INFINITY;
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
        // ---- values
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float a = alpha[h];
#pragma unroll
            for (int d = 0; d < 4; ++d) acc[h][d] *= a;
        }
#pragma unroll 4
        for (int i = 0; i < 32; ++i) {
            const int key = t0 + warp * 32 + i;
            if (key >= k_end) break;
            uint2 u = *reinterpret_cast<const uint2 *>(V + size_t(key) * AD_D + lane * 4);
            const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&u);
            float2 f0 = __bfloat1622float2(u2[0]), f1 = __bfloat1622float2(u2[1]);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = S[warp * 32 + i][h];
                acc[h][0] += pr * f0.x;
                acc[h][1] += pr * f0.y;
                acc[h][2] += pr * f1.x;
                acc[h][3] += pr * f1.y;
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
    const size_t base = (size_t(b) * p.Hkv + kvh) * p.splits * G;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) {
        const int h = i / AD_D, d = i % AD_D;
        float M = -INFINITY;
        for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.ws_ml[(base + size_t(s) * G + h) * 2]);
        float L = 0.f, O = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float ms = p.ws_ml[(base + size_t(s) * G + h) * 2];
            if (ms == -INFINITY) continue;
            const float f = exp2f(ms - M);
            L += p.ws_ml[(base + size_t(s) * G + h) * 2 + 1] * f;
            O += p.ws_o[(base + size_t(s) * G + h) * AD_D + d] * f;
        }
        p.out[(size_t(b) * p.Hq + size_t(kvh) * G + h) * AD_D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
    }
    if (threadIdx.x == 0) p.counters[b * p.Hkv + kvh] = 0;
}

}  // namespace xt

using namespace xt;

extern "C" int xt_attn_decode(const AttnDecodeParams *pp, int B, cudaStream_t stream) {
    AttnDecodeParams p = *pp;
    const int G = p.Hq / p.Hkv;
    if (p.Hq % p.Hkv) return -2;
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
