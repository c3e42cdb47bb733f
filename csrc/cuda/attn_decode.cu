// GQA decode attention over a contiguous BF16 KV cache [B, Hkv, L, D=128], split over the keys (flash-decoding).
//
// Grid (splits, Hkv, B), 8 warps. A CTA takes the G = Hq/Hkv query heads of one KV head and a fixed slice of the cache
// (L / splits keys, cut at the sequence length), walked in tiles of 256 keys with an online softmax:
//   scores  each warp takes 32 keys, one per lane: the lane loads its key's 256-byte row (16 independent 16-byte
//           loads in flight) and forms the G head dots against the pre-scaled queries in shared memory (broadcast
//           reads), so no cross-lane reduction is needed.
//   softmax one warp per head: tile max, running max and sum, exp2 in place.
//   values  lane l accumulates dims 4l..4l+3 of all G heads; the warp's 32 value rows are loaded (8 bytes per lane)
//           before the softmax, so the whole tile costs two memory round trips.
// Each split writes its unnormalized output, max and sum to a workspace; the last CTA of a (batch, KV head) to finish
// merges the splits (an arrival counter that it resets), so one launch does the whole step and the grid shape does not
// depend on the sequence length (graph capture). Sequence lengths are read from device memory.
// Reference parity: the reference leaves dense decode attention to SGLang's backends; this kernel is the dense
// attention of the Qwen3-style config (GQA 32/4, head dim 128).
#include "common.cuh"
#include "params.h"

namespace xt {

constexpr int AD_WARPS = 8;
constexpr int AD_TILE = 32 * AD_WARPS;   // keys per tile: one per lane
constexpr int AD_D = 128;
constexpr int AD_MAX_SPLITS = 64;

template <int G>
struct AdSmem {   // dynamic shared memory layout
    static constexpr size_t S = size_t(AD_TILE) * G * 4;          // scores of a tile [key][head]
    static constexpr size_t RED = size_t(AD_WARPS) * G * AD_D * 4;  // cross-warp reduction [warp][head][dim]
    static constexpr size_t BUF = S > RED ? S : RED;
    static constexpr size_t Q = size_t(G) * AD_D * 4;
    static constexpr size_t BYTES = BUF + Q + 3 * G * 4 + AD_MAX_SPLITS * G * 4 + 64;
};

template <int G>
__global__ void __launch_bounds__(AD_WARPS * 32) attn_decode_kernel(AttnDecodeParams p) {
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    extern __shared__ __align__(16) uint8_t dsm[];
    float *buf = reinterpret_cast<float *>(dsm);
    float(&S)[AD_TILE][G] = *reinterpret_cast<float(*)[AD_TILE][G]>(buf);
    float(&red)[AD_WARPS][G][AD_D] = *reinterpret_cast<float(*)[AD_WARPS][G][AD_D]>(buf);
    float(&qs)[G][AD_D] = *reinterpret_cast<float(*)[G][AD_D]>(dsm + AdSmem<G>::BUF);
    float *m_run = reinterpret_cast<float *>(dsm + AdSmem<G>::BUF + AdSmem<G>::Q);
    float *l_run = m_run + G, *alpha = l_run + G;
    float(&wsplit)[AD_MAX_SPLITS][G] = *reinterpret_cast<float(*)[AD_MAX_SPLITS][G]>(alpha + G);
    __shared__ bool last;

    // the split's key range is a fixed slice of the cache, so the first tile's K loads need no sequence length
    const int chunk = (p.L + p.splits - 1) / p.splits;
    const int k_begin = split * chunk;
    const size_t head_off = (size_t(b) * p.Hkv + kvh) * p.L;
    const __nv_bfloat16 *K = p.kc + head_off * AD_D;
    const __nv_bfloat16 *V = p.vc + head_off * AD_D;

    const __nv_bfloat16 *qb = p.q + (size_t(b) * p.Hq + size_t(kvh) * G) * AD_D;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) qs[i / AD_D][i % AD_D] = __bfloat162float(qb[i]) * p.scale_log2;
    if (threadIdx.x < G) {
        m_run[threadIdx.x] = -INFINITY;
        l_run[threadIdx.x] = 0.f;
    }
    const int N = p.seqlens[b];
    const int k_end = min(N, k_begin + chunk);
    __syncthreads();
    float acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;

    for (int t0 = k_begin; t0 < k_end; t0 += AD_TILE) {
        // ---- scores: one key per lane, its whole 256-byte row in flight at once
        {
            const int key = t0 + warp * 32 + lane;
            const bool valid = key < k_end;
            const uint4 *kr = reinterpret_cast<const uint4 *>(K + size_t(valid ? key : t0) * AD_D);
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
        // ---- this warp's 32 value rows (8 bytes per lane each) in flight while the softmax runs
        const int nk = max(0, min(32, k_end - (t0 + warp * 32)));
        uint2 vv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int key = t0 + warp * 32 + min(i, max(nk - 1, 0));
            vv[i] = *reinterpret_cast<const uint2 *>(V + size_t(key) * AD_D + lane * 4);
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
        // ---- values: lane owns dims 4l..4l+3 of every head
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float a = alpha[h];
#pragma unroll
            for (int d = 0; d < 4; ++d) acc[h][d] *= a;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (i >= nk) break;
            const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&vv[i]);
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
    // ---- the last split to arrive merges (arrival counter, reset by the merging CTA)
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
    float *mls = buf;
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
    // four consecutive dims per thread; every split's 16-byte load issued before any is used (up to 16 splits)
    const size_t stride4 = size_t(G) * AD_D / 4;
    for (int i = threadIdx.x * 4; i < G * AD_D; i += blockDim.x * 4) {
        const int h = i / AD_D;
        const float4 *src = reinterpret_cast<const float4 *>(p.ws_o + base * AD_D + i);
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < p.splits; s0 += 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = s0 + j < p.splits ? __ldcg(src + (s0 + j) * stride4) : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float wgt = s0 + j < p.splits ? wsplit[s0 + j][h] : 0.f;
                O.x += v[j].x * wgt;
                O.y += v[j].y * wgt;
                O.z += v[j].z * wgt;
                O.w += v[j].w * wgt;
            }
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
    if (p.Hq % p.Hkv || p.splits < 1 || p.splits > AD_MAX_SPLITS) return -2;
    dim3 grid(p.splits, p.Hkv, B);
#define XT_AD(GG)                                                                                                  \
    case GG: {                                                                                                     \
        static bool attr = false;                                                                                  \
        const int smem = int(AdSmem<GG>::BYTES);                                                                   \
        if (!attr) {                                                                                               \
            cudaFuncSetAttribute(attn_decode_kernel<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);       \
            attr = true;                                                                                           \
        }                                                                                                          \
        attn_decode_kernel<GG><<<grid, AD_WARPS * 32, smem, stream>>>(p);                                          \
        break;                                                                                                     \
    }
    switch (G) {
        XT_AD(1) XT_AD(2) XT_AD(4) XT_AD(8) XT_AD(16)
        default: return -3;
    }
#undef XT_AD
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
