// DSA-style sparse attention selection (DeepSeek sparse attention's "lightning indexer"), decode path, sm_100a:
//
//   dsa_key_write     one warp per new token: its 128-dim index key -> FP8 E4M3 with one FP32 scale per token
//                     (amax / 448), 132 bytes per token.
//   dsa_index_decode  score of every cached key s of a query t: I(t, s) = sum_h w[t, h] * relu(q[t, h] . k[s]),
//                     64 heads of dim 128 (the heads share the key, as in MQA). Grid (blocks of 64 keys, queries);
//                     4 threads per key, each with 16 heads, the queries in shared memory (broadcast reads); keys past
//                     the query's length score -inf.
//   topk_rows         the K largest scores of each row -> their indices in ascending order (-1 padding when a row has
//                     fewer than K finite scores). One CTA per row: a 4-pass radix select on the order-preserving
//                     integer image of the floats finds the K-th largest value, then one ordered compaction pass (block
//                     scans) writes the elements above it and, in index order, as many equal to it as are needed --
//                     so the selected set and its order do not depend on thread timing.
// Reference parity: the reference drives DeepSeek V4's indexer through SGLang and its packs (xtier/packs/
// deepseek_v4/paged_indexer.py:1-13 scores a decode step's compressed index keys and selects with a top-k kernel;
// xtier/packs/qwen4_exp/qsa_prefill.py:1-12 the ReLU head-sum MQA logits).
#include "common.cuh"
#include "params.h"

namespace xt {

constexpr int IDX_HEADS = 64, IDX_DIM = 128;

__global__ void __launch_bounds__(256) dsa_key_write_kernel(const __nv_bfloat16 *__restrict__ k, const int64_t *slot,
                                                            uint8_t *codes, float *kscale, int T) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const __nv_bfloat16 *x = k + size_t(warp) * IDX_DIM;
    float v[4];
    const uint2 u = reinterpret_cast<const uint2 *>(x)[lane];
    const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
    const float2 f0 = __bfloat1622float2(b[0]), f1 = __bfloat1622float2(b[1]);
    v[0] = f0.x;
    v[1] = f0.y;
    v[2] = f1.x;
    v[3] = f1.y;
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = warp_max(amax);
    const float sc = amax > 0.f ? amax / 448.f : 1.f;
    const float inv = 1.f / sc;
    uint16_t lo, hi;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(lo) : "f"(v[1] * inv), "f"(v[0] * inv));
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(hi) : "f"(v[3] * inv), "f"(v[2] * inv));
    const size_t s = size_t(slot[warp]);
    reinterpret_cast<uint32_t *>(codes + s * IDX_DIM)[lane] = uint32_t(lo) | (uint32_t(hi) << 16);
    if (lane == 0) kscale[s] = sc;
}

// q [Q, 64, 128] bf16, w [Q, 64] f32, codes [slots, 128] e4m3, kscale [slots] f32; query t reads slots
// base[t] .. base[t] + len[t] - 1; scores [Q, max_len] f32.
__global__ void __launch_bounds__(256) dsa_index_decode_kernel(const __nv_bfloat16 *__restrict__ q,
                                                               const float *__restrict__ w,
                                                               const uint8_t *__restrict__ codes,
                                                               const float *__restrict__ kscale,
                                                               const int64_t *__restrict__ base,
                                                               const int32_t *__restrict__ len, float *scores,
                                                               int max_len) {
    __shared__ __align__(16) float qs[IDX_HEADS][IDX_DIM];
    __shared__ float ws[IDX_HEADS];
    const int t = blockIdx.y;
    for (int i = threadIdx.x; i < IDX_HEADS * IDX_DIM; i += blockDim.x)
        qs[i / IDX_DIM][i % IDX_DIM] = __bfloat162float(q[size_t(t) * IDX_HEADS * IDX_DIM + i]);
    if (threadIdx.x < IDX_HEADS) ws[threadIdx.x] = w[size_t(t) * IDX_HEADS + threadIdx.x];
    __syncthreads();
    const int key = blockIdx.x * 64 + (threadIdx.x >> 2), hq = threadIdx.x & 3;   // 4 threads per key, 16 heads each
    const int n = len[t];
    const bool valid = key < n && key < max_len;
    float part = 0.f;
    if (valid) {
        const uint8_t *kr = codes + (size_t(base[t]) + key) * IDX_DIM;
        float acc[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) acc[h] = 0.f;
#pragma unroll
        for (int c = 0; c < IDX_DIM / 16; ++c) {
            const uint4 u = reinterpret_cast<const uint4 *>(kr)[c];
            const uint16_t *p2 = reinterpret_cast<const uint16_t *>(&u);
            float kf[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float2 f = e4m3x2_to_f2(p2[i]);
                kf[2 * i] = f.x;
                kf[2 * i + 1] = f.y;
            }
#pragma unroll
            for (int h = 0; h < 16; ++h) {
                const float *qr = &qs[hq * 16 + h][c * 16];
                float a = acc[h];
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                    const float4 qv = *reinterpret_cast<const float4 *>(qr + i);
                    a = fmaf(qv.x, kf[i], fmaf(qv.y, kf[i + 1], fmaf(qv.z, kf[i + 2], fmaf(qv.w, kf[i + 3], a))));
                }
                acc[h] = a;
            }
        }
        const float ks = kscale[size_t(base[t]) + key];
#pragma unroll
        for (int h = 0; h < 16; ++h) part += ws[hq * 16 + h] * fmaxf(acc[h] * ks, 0.f);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (hq == 0 && key < max_len) scores[size_t(t) * max_len + key] = valid ? part : -INFINITY;
}

// order-preserving image of a float: larger float -> larger unsigned (NaN never occurs here)
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int TK_THREADS = 1024;

// exclusive scan of v over the block; returns this thread's prefix, total in *tot
__device__ int block_scan(int v, int *warp_sums, int *tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = lane < TK_THREADS / 32 ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;   // inclusive
    }
    __syncthreads();
    const int before = (warp ? warp_sums[warp - 1] : 0) + x - v;
    *tot = warp_sums[TK_THREADS / 32 - 1];
    __syncthreads();
    return before;
}

__global__ void __launch_bounds__(TK_THREADS) topk_rows_kernel(const float *__restrict__ scores, int n, int K,
                                                               int32_t *__restrict__ out) {
    __shared__ int hist[256];
    __shared__ int warp_sums[32];
    __shared__ uint32_t prefix_s;
    __shared__ int need_s;
    const int row = blockIdx.x;
    const float *x = scores + size_t(row) * n;
    int32_t *o = out + size_t(row) * K;
    // radix select of the K-th largest key among finite scores
    uint32_t prefix = 0;
    int need = K;
    int finite = 0;
    for (int i = threadIdx.x; i < n; i += TK_THREADS) finite += x[i] > -INFINITY;
    int tot;
    block_scan(finite, warp_sums, &tot);
    const bool all = tot <= K;
    if (!all) {
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            const uint32_t mask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
            for (int i = threadIdx.x; i < 256; i += TK_THREADS) hist[i] = 0;
            __syncthreads();
            for (int i = threadIdx.x; i < n; i += TK_THREADS) {
                const float v = x[i];
                if (v == -INFINITY) continue;
                const uint32_t k = fkey(v);
                if ((k & mask) == (prefix & mask)) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
            }
            __syncthreads();
            if (threadIdx.x == 0) {   // walk the buckets from the largest
                int acc = 0, b = 255;
                for (; b > 0; --b) {
                    if (acc + hist[b] >= need) break;
                    acc += hist[b];
                }
                prefix_s = prefix | (uint32_t(b) << shift);
                need_s = need - acc;
            }
            __syncthreads();
            prefix = prefix_s;
            need = need_s;
            __syncthreads();
        }
    }
    // ordered compaction: keys above the threshold, then `need` of the keys equal to it, in index order
    const uint32_t thr = prefix;
    int gt_before = 0, eq_before = 0;
    for (int c0 = 0; c0 < n; c0 += TK_THREADS) {
        const int i = c0 + threadIdx.x;
        const float v = i < n ? x[i] : -INFINITY;
        const bool fin = v > -INFINITY;
        const uint32_t k = fin ? fkey(v) : 0u;
        const int gt = all ? int(fin) : int(fin && k > thr);
        const int eq = all ? 0 : int(fin && k == thr);
        int t_gt, t_eq;
        const int p_gt = block_scan(gt, warp_sums, &t_gt);
        const int p_eq = block_scan(eq, warp_sums, &t_eq);
        const int eq_rank = eq_before + p_eq;
        const bool take_eq = eq && eq_rank < need;
        // output position: elements taken before i in index order
        const int taken_before_gt = gt_before + p_gt;
        const int taken_before_eq = min(eq_before + p_eq, need);
        const int pos = taken_before_gt + taken_before_eq;
        if ((gt || take_eq) && pos < K) o[pos] = i;
        gt_before += t_gt;
        eq_before += t_eq;
    }
    const int taken = gt_before + (all ? 0 : min(eq_before, need));
    for (int i = taken + threadIdx.x; i < K; i += TK_THREADS) o[i] = -1;
}

}  // namespace xt

using namespace xt;

extern "C" {

int xt_dsa_key_write(const void *k, const int64_t *slot, void *codes, float *kscale, int T, cudaStream_t stream) {
    if (T <= 0) return 0;
    dsa_key_write_kernel<<<(T + 7) / 8, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(k), slot,
                                                          static_cast<uint8_t *>(codes), kscale, T);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_dsa_index_decode(const void *q, const float *w, const void *codes, const float *kscale, const int64_t *base,
                        const int32_t *len, float *scores, int Q, int max_len, cudaStream_t stream) {
    if (Q <= 0 || max_len <= 0) return -2;
    dim3 grid((max_len + 63) / 64, Q);
    dsa_index_decode_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(q), w,
                                                      static_cast<const uint8_t *>(codes), kscale, base, len, scores,
                                                      max_len);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_topk_rows(const float *scores, int rows, int n, int K, int32_t *out, cudaStream_t stream) {
    if (rows <= 0 || n <= 0 || K <= 0) return -2;
    topk_rows_kernel<<<rows, TK_THREADS, 0, stream>>>(scores, n, K, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
