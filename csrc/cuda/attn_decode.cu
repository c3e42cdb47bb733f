// GQA decode attention over a contiguous BF16 KV cache [B, Hkv, L, D=128], split over the keys (flash-decoding).
//
// Grid (splits, Hkv, B), 8 warps. A CTA takes the G = Hq/Hkv query heads of one KV head and 1/splits of the sequence's
// keys (the split is cut from the sequence length read on the device, so every split has work and the grid does not
// depend on the length: graph capture), walked in tiles of 64 keys with an online softmax:
//   scores  a warp takes 8 keys, 4 lanes per key: each lane loads 64 bytes of its key's row (4 independent 16-byte
//           loads) and forms the partial dots of its 32 dims with the G pre-scaled queries (shared-memory broadcast
//           reads); two shuffles finish each dot.
//   softmax one warp per head: tile max, running max and sum, exp2 in place.
//   values  the warp's 8 value rows are loaded before the softmax (8 bytes per lane each); lane l accumulates dims
//           4l..4l+3 of every head over its warp's keys.
// With 64-key tiles a 2K-token sequence spreads over ~36 splits x Hkv CTAs, so the step costs about one memory round
// trip plus a short dependent chain per CTA. Each split writes its unnormalized output, max and sum to a workspace;
// the last CTA of a (batch, KV head) to finish merges the splits (an arrival counter that it resets), so one launch
// does the whole step.
// Reference parity: the reference leaves dense decode attention to SGLang's backends; this kernel is the dense
// attention of the Qwen3-style config (GQA 32/4, head dim 128).
#include "common.cuh"
#include "params.h"
#include "tc_common.cuh"
#include <stdlib.h>

namespace xt {

constexpr int AD_WARPS = 8;
constexpr int AD_KPW = 8;                    // keys per warp and tile
constexpr int AD_TILE = AD_KPW * AD_WARPS;   // keys per tile
constexpr int AD_D = 128;
constexpr int AD_MAX_SPLITS = 64;

template <int G>
struct AdSmem {   // dynamic shared memory layout
    static constexpr size_t S = size_t(AD_TILE) * G * 4;            // scores of a tile [key][head]
    static constexpr size_t RED = size_t(AD_WARPS) * G * AD_D * 4;  // cross-warp reduction [warp][head][dim]
    static constexpr size_t MERGE = size_t(AD_MAX_SPLITS) * G * 2 * 4;
    static constexpr size_t BUF0 = S > RED ? S : RED;
    static constexpr size_t BUF = BUF0 > MERGE ? BUF0 : MERGE;
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
    pdl_wait();
    pdl_trigger();

    const size_t head_off = (size_t(b) * p.Hkv + kvh) * p.L;
    const __nv_bfloat16 *K = p.kc + head_off * AD_D;
    const __nv_bfloat16 *V = p.vc + head_off * AD_D;
    const __nv_bfloat16 *qb = p.q + (size_t(b) * p.Hq + size_t(kvh) * G) * AD_D;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) qs[i / AD_D][i % AD_D] = __bfloat162float(qb[i]) * p.scale_log2;
    if (threadIdx.x < G) {
        m_run[threadIdx.x] = -INFINITY;
        l_run[threadIdx.x] = 0.f;
    }
    const int N = min(p.seqlens[b], p.L);
    const int chunk = (((N + p.splits - 1) / p.splits) + 7) & ~7;
    const int k_begin = split * chunk;
    const int k_end = min(N, k_begin + chunk);
    __syncthreads();
    float acc[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[h][d] = 0.f;
    const int kq = lane >> 2, qd = lane & 3;   // key of the warp's 8, quarter of the 128 dims

    for (int t0 = k_begin; t0 < k_end; t0 += AD_TILE) {
        const int kw = t0 + warp * AD_KPW;   // first key of this warp
        // ---- loads: 64 bytes of one key row per lane, and the warp's 8 value rows (8 bytes per lane each)
        const int key = kw + kq;
        const bool valid = key < k_end;
        const uint4 *kr = reinterpret_cast<const uint4 *>(K + size_t(valid ? key : k_begin) * AD_D + qd * 32);
        uint4 kv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) kv[c] = kr[c];
        uint2 vv[AD_KPW];
#pragma unroll
        for (int i = 0; i < AD_KPW; ++i) {
            const int kvk = min(kw + i, k_end - 1);
            vv[i] = *reinterpret_cast<const uint2 *>(V + size_t(max(kvk, k_begin)) * AD_D + lane * 4);
        }
        // ---- scores
        {
            float s[G];
#pragma unroll
            for (int h = 0; h < G; ++h) s[h] = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&kv[c]);
                float kf[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(k2[i]);
                    kf[2 * i] = f.x;
                    kf[2 * i + 1] = f.y;
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(&qs[h][qd * 32 + c * 8]);
                    const float4 q1 = *reinterpret_cast<const float4 *>(&qs[h][qd * 32 + c * 8 + 4]);
                    s[h] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                            q1.z * kf[6] + q1.w * kf[7];
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) {
                s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);
                s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
            }
            if (qd == 0) {
#pragma unroll
                for (int h = 0; h < G; ++h) S[warp * AD_KPW + kq][h] = valid ? s[h] : -INFINITY;
            }
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
                const float e = (m_new == -INFINITY) ? 0.f : exp2f(S[i][h] - m_new);
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
        // ---- values: lane owns dims 4l..4l+3 of every head, over its warp's 8 keys
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float a = alpha[h];
#pragma unroll
            for (int d = 0; d < 4; ++d) acc[h][d] *= a;
        }
#pragma unroll
        for (int i = 0; i < AD_KPW; ++i) {
            const __nv_bfloat162 *u2 = reinterpret_cast<const __nv_bfloat162 *>(&vv[i]);
            const float2 f0 = __bfloat1622float2(u2[0]), f1 = __bfloat1622float2(u2[1]);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = S[warp * AD_KPW + i][h];   // 0 for keys past the end (score -inf)
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


// ---------------------------------------------------------------------------------------------------------------
// Tensor-core variant for query groups of 8 or 16 heads (mma.sync m16n8k16, BF16 in, FP32 accumulate).
//
// The G heads of a KV head are the 16 rows of the MMA's A operand (rows past G are zero). A CTA of AM_WARPS warps
// takes one split of the keys; every warp walks its own 16-key blocks (block i of the split goes to warp i % 4) with
// its own online softmax, so no CTA-wide barrier sits in the key loop:
//   S = Q K^T   the contraction over the 128 dims is permuted (the same permutation for Q and K, so the dot products
//               are unchanged) such that thread (g, t) of the warp needs dims 32t..32t+31 of key g of each 8-key
//               tile: four 16-byte global loads per key tile, the 16 fragments of Q held in registers all along;
//   softmax     per head row: two shuffles for the max, the sum kept per thread and reduced once at the end;
//   O += P V    P comes straight from the S accumulators (re-packed as the A operand); V goes through shared memory
//               (cp.async, 16-byte chunks, XOR-swizzled by key) and ldmatrix.trans builds its fragments.
// The next block's K fragments and V tile are in flight while the current block computes (double buffer). At the
// end the CTA merges its warps in shared memory and writes the split's partial; the last split of a (batch, KV head)
// merges the splits, as in the kernel above.
constexpr int AM_WARPS = 4;
constexpr int AM_KB = 16;   // keys per warp block

template <int G>
struct AmSmem {
    static constexpr size_t V = size_t(AM_WARPS) * 2 * AM_KB * AD_D * 2;   // 32 KB: per warp, two V tiles
    static constexpr size_t O = size_t(AM_WARPS) * G * AD_D * 4;          // warp partials
    static constexpr size_t ML = size_t(AM_WARPS) * G * 2 * 4;
    static constexpr size_t MERGE = size_t(AD_MAX_SPLITS) * G * 2 * 4 + size_t(AD_MAX_SPLITS) * G * 4;
    static constexpr size_t BYTES = V + (O > MERGE ? O : MERGE) + ML + 64;
};

XT_DEV void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

XT_DEV uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

XT_DEV uint4 ldg_v4(const void *p) { return *reinterpret_cast<const uint4 *>(p); }

// one warp's block: K fragments of keys [kb, kb + 16) (clamped to `last`) into registers, V tile into shared memory
XT_DEV void am_load(const __nv_bfloat16 *K, const __nv_bfloat16 *V, int kb, int last, int lane, uint4 (&kf)[2][4],
                    uint8_t *vt) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int key = min(kb + j * 8 + g, last);
        const uint8_t *row = reinterpret_cast<const uint8_t *>(K + size_t(key) * AD_D) + t * 64;
#pragma unroll
        for (int c = 0; c < 4; ++c) kf[j][c] = ldg_v4(row + c * 16);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int i = lane + 32 * r;           // chunk of the 16 x 16 chunks of the tile
        const int key = i >> 4, ch = i & 15;
        const uint8_t *src = reinterpret_cast<const uint8_t *>(V + size_t(min(kb + key, last)) * AD_D) + ch * 16;
        const uint32_t dst = tc::smem_u32(vt + key * 256 + ((ch ^ (key & 7)) << 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <int G>
XT_DEV void am_block(const uint32_t (&qa)[8][4], const uint4 (&kf)[2][4], const uint8_t *vt, int kb, int kend,
                     float scale_log2, int lane, float (&o)[16][4], float (&m)[2], float (&l)[2]) {
    const int t = lane & 3;
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
        const uint32_t *kw = reinterpret_cast<const uint32_t *>(&kf[j][0]);
#pragma unroll
        for (int s = 0; s < 8; ++s) mma_bf16_16816(sc[j], qa[s][0], qa[s][1], qa[s][2], qa[s][3], kw[2 * s], kw[2 * s + 1]);
    }
    // scale, mask, online softmax per row (r = 0: head g, r = 1: head g + 8)
    uint32_t pa[4];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (r == 1 && G <= 8) {
            pa[1] = pa[3] = 0u;
            continue;
        }
        float v[4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = kb + j * 8 + t * 2 + e;
                v[j * 2 + e] = key < kend ? sc[j][r * 2 + e] * scale_log2 : -INFINITY;
            }
        float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m[r], mx);
        const float alpha = mn == -INFINITY ? 1.f : exp2f(m[r] - mn);
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pr[i] = v[i] == -INFINITY ? 0.f : exp2f(v[i] - mn);
        l[r] = l[r] * alpha + pr[0] + pr[1] + pr[2] + pr[3];
        m[r] = mn;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            o[nt][r * 2] *= alpha;
            o[nt][r * 2 + 1] *= alpha;
        }
        pa[r] = pack_bf16(pr[0], pr[1]);       // keys t*2, t*2+1 of tile 0
        pa[r + 2] = pack_bf16(pr[2], pr[3]);   // keys 8+t*2, 8+t*2+1 of tile 1
    }
    // O += P V: V^T fragments by ldmatrix.trans from the swizzled tile
    const int key = (lane & 7) + ((lane >> 3) & 1) * 8, half = lane >> 4;
#pragma unroll
    for (int nt = 0; nt < 16; nt += 2) {
        const int ch = nt + half;   // 16-byte chunk = 8 dims
        const uint32_t addr = tc::smem_u32(vt + key * 256 + ((ch ^ (key & 7)) << 4));
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                     : "r"(addr));
        mma_bf16_16816(o[nt], pa[0], pa[1], pa[2], pa[3], b0, b1);
        mma_bf16_16816(o[nt + 1], pa[0], pa[1], pa[2], pa[3], b2, b3);
    }
}

template <int G>
__global__ void __launch_bounds__(AM_WARPS * 32) attn_decode_mma_kernel(AttnDecodeParams p) {
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    extern __shared__ __align__(128) uint8_t dsm[];
    uint8_t *vtiles = dsm + size_t(warp) * 2 * AM_KB * 256;
    float(&os)[AM_WARPS][G][AD_D] = *reinterpret_cast<float(*)[AM_WARPS][G][AD_D]>(dsm + AmSmem<G>::V);
    float(&mls)[AM_WARPS][G][2] =
        *reinterpret_cast<float(*)[AM_WARPS][G][2]>(dsm + AmSmem<G>::V + (AmSmem<G>::O > AmSmem<G>::MERGE
                                                                              ? AmSmem<G>::O
                                                                              : AmSmem<G>::MERGE));
    __shared__ bool last;
    pdl_wait();
    pdl_trigger();

    const size_t head_off = (size_t(b) * p.Hkv + kvh) * p.L;
    const __nv_bfloat16 *K = p.kc + head_off * AD_D;
    const __nv_bfloat16 *V = p.vc + head_off * AD_D;
    const __nv_bfloat16 *qb = p.q + (size_t(b) * p.Hq + size_t(kvh) * G) * AD_D;
    // Q fragments (rows g and g + 8 of the permuted 16 x 128 operand): dims 32t..32t+31, words 2s / 2s+1 per step
    uint32_t qa[8][4];
    {
        uint4 q0[4], q1[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            q0[c] = g < G ? ldg_v4(reinterpret_cast<const uint8_t *>(qb + size_t(g) * AD_D) + t * 64 + c * 16)
                          : make_uint4(0, 0, 0, 0);
            q1[c] = g + 8 < G ? ldg_v4(reinterpret_cast<const uint8_t *>(qb + size_t(g + 8) * AD_D) + t * 64 + c * 16)
                              : make_uint4(0, 0, 0, 0);
        }
        const uint32_t *w0 = reinterpret_cast<const uint32_t *>(q0), *w1 = reinterpret_cast<const uint32_t *>(q1);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            qa[s][0] = w0[2 * s];
            qa[s][1] = w1[2 * s];
            qa[s][2] = w0[2 * s + 1];
            qa[s][3] = w1[2 * s + 1];
        }
    }
    const int N = min(p.seqlens[b], p.L);
    const int chunk = (((N + p.splits - 1) / p.splits) + 7) & ~7;
    const int k_begin = split * chunk;
    const int k_end = min(N, k_begin + chunk);
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    const int last_key = max(k_end - 1, 0);
    const int step = AM_WARPS * AM_KB;
    int kb = k_begin + warp * AM_KB;
    if (kb < k_end) {
        uint4 ka[2][4], kn[2][4];
        am_load(K, V, kb, last_key, lane, ka, vtiles);
        for (;;) {
            const int nb = kb + step;
            if (nb < k_end) am_load(K, V, nb, last_key, lane, kn, vtiles + AM_KB * 256);
            if (nb < k_end)
                asm volatile("cp.async.wait_group 1;\n" ::: "memory");
            else
                asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            __syncwarp();
            am_block<G>(qa, ka, vtiles, kb, k_end, p.scale_log2, lane, o, m, l);
            __syncwarp();
            if (nb >= k_end) break;
            kb = nb;
            const int nb2 = kb + step;
            if (nb2 < k_end) am_load(K, V, nb2, last_key, lane, ka, vtiles);
            if (nb2 < k_end)
                asm volatile("cp.async.wait_group 1;\n" ::: "memory");
            else
                asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            __syncwarp();
            am_block<G>(qa, kn, vtiles + AM_KB * 256, kb, k_end, p.scale_log2, lane, o, m, l);
            __syncwarp();
            if (nb2 >= k_end) break;
            kb = nb2;
        }
    }
    // ---- this warp's rows to shared memory (sums reduced over the row's four threads)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
        const int h = g + r * 8;
        if (h < G) {
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
                os[warp][h][nt * 8 + t * 2] = o[nt][r * 2];
                os[warp][h][nt * 8 + t * 2 + 1] = o[nt][r * 2 + 1];
            }
            if (t == 0) {
                mls[warp][h][0] = m[r];
                mls[warp][h][1] = l[r];
            }
        }
    }
    __syncthreads();
    // ---- merge the warps: this split's unnormalized output, max and sum
    const size_t part = ((size_t(b) * p.Hkv + kvh) * p.splits + split) * G;
    for (int i = threadIdx.x; i < G * AD_D; i += blockDim.x) {
        const int h = i / AD_D, d = i % AD_D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < AM_WARPS; ++w) M = fmaxf(M, mls[w][h][0]);
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < AM_WARPS; ++w) {
            const float mw = mls[w][h][0];
            acc += mw == -INFINITY ? 0.f : os[w][h][d] * exp2f(mw - M);
        }
        p.ws_o[part * AD_D + i] = acc;
    }
    if (threadIdx.x < G) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < AM_WARPS; ++w) M = fmaxf(M, mls[w][h][0]);
        float L = 0.f;
        for (int w = 0; w < AM_WARPS; ++w) {
            const float mw = mls[w][h][0];
            L += mw == -INFINITY ? 0.f : mls[w][h][1] * exp2f(mw - M);
        }
        p.ws_ml[(part + h) * 2] = M;
        p.ws_ml[(part + h) * 2 + 1] = L;
    }
    // ---- the last split to arrive merges (arrival counter, reset by the merging CTA)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.counters[b * p.Hkv + kvh], 1u);
        last = prev == unsigned(p.splits) - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    float *msp = reinterpret_cast<float *>(dsm + AmSmem<G>::V);         // [splits][G][2]
    float *wsp = msp + AD_MAX_SPLITS * G * 2;                            // [splits][G]
    const size_t base = (size_t(b) * p.Hkv + kvh) * p.splits * G;
    for (int i = threadIdx.x; i < p.splits * G * 2; i += blockDim.x) msp[i] = __ldcg(p.ws_ml + base * 2 + i);
    __syncthreads();
    if (threadIdx.x < G) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int s2 = 0; s2 < p.splits; ++s2) M = fmaxf(M, msp[(s2 * G + h) * 2]);
        float L = 0.f;
        for (int s2 = 0; s2 < p.splits; ++s2) {
            const float ms = msp[(s2 * G + h) * 2];
            const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
            wsp[s2 * G + h] = f;
            L += msp[(s2 * G + h) * 2 + 1] * f;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int s2 = 0; s2 < p.splits; ++s2) wsp[s2 * G + h] *= inv;
    }
    __syncthreads();
    const size_t stride4 = size_t(G) * AD_D / 4;
    for (int i = threadIdx.x * 4; i < G * AD_D; i += blockDim.x * 4) {
        const int h = i / AD_D;
        const float4 *src = reinterpret_cast<const float4 *>(p.ws_o + base * AD_D + i);
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < p.splits; s0 += 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                v[j] = s0 + j < p.splits ? __ldcg(src + (s0 + j) * stride4) : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float wgt = s0 + j < p.splits ? wsp[(s0 + j) * G + h] : 0.f;
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
    static const bool legacy = [] {   // XTIER_ATTN_CUDA_CORES=1: the CUDA-core kernel for every group size
        const char *v = getenv("XTIER_ATTN_CUDA_CORES");
        return v && atoi(v) != 0;
    }();
    if (!legacy && (G == 8 || G == 16)) {
#define XT_AM(GG)                                                                                                  \
        {                                                                                                          \
            const int smem = int(AmSmem<GG>::BYTES);                                                               \
            xt_smem_optin(attn_decode_mma_kernel<GG>, smem);                                                       \
            if (xt_launch(attn_decode_mma_kernel<GG>, grid, dim3(AM_WARPS * 32), smem, stream, p) != cudaSuccess)  \
                return -1;                                                                                         \
        }
        if (G == 8) XT_AM(8) else XT_AM(16)
#undef XT_AM
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
#define XT_AD(GG)                                                                                                  \
    case GG: {                                                                                                     \
        const int smem = int(AdSmem<GG>::BYTES);                                                                   \
        xt_smem_optin(attn_decode_kernel<GG>, smem);                                                               \
        if (xt_launch(attn_decode_kernel<GG>, grid, dim3(AD_WARPS * 32), smem, stream, p) != cudaSuccess)           \
            return -1;                                                                                             \
        break;                                                                                                     \
    }
    switch (G) {
        XT_AD(1) XT_AD(2) XT_AD(4) XT_AD(8) XT_AD(16)
        default: return -3;
    }
#undef XT_AD
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ================================================================================================================
// xt_attn_decode_noalloc: the decode attention above for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference. Some callers cannot call cudaMalloc: code that runs inside
// another framework's memory pool with no allocator handed to it, plugins whose host process forbids allocation after
// start-up, and real-time serving loops that must never hit the driver allocator. xt_attn_decode needs a workspace for
// the split partials (output, max and sum per split and head) and arrival counters; here that workspace is a
// file-scope device array of fixed size, so the caller passes only the inputs and the output.
//
//  * Limit: B * Hkv * splits * G * (128 + 2) floats must fit in XT_AD_NOALLOC_FLOATS (512 Ki floats, 2 MiB), and
//    B * Hkv must not exceed XT_AD_NOALLOC_COUNTERS (4096); larger calls return XT_AD_NOALLOC_TOO_BIG and the text of
//    xt_attn_decode_noalloc_error() says which limit was exceeded. Every GPU that loads this library holds the 2 MiB
//    (plus 16 KiB of counters) until the process exits.
//  * Set-up: the first call on a device looks up the array's device address with cudaGetSymbolAddress (and sets the
//    kernels' shared-memory attribute) with that device current. Make that first call before any stream capture.
//  * The array is shared by every call and keeps the last call's contents. Each call clears the arrival counters it
//    uses (cudaMemsetAsync on its stream) before the kernel; calls that overlap on the GPU (different streams, or
//    different host threads) race on the array and give wrong results: serialize them.
//  * The call allocates nothing: no cudaMalloc, no cudaFree, no library routine that allocates.
// ================================================================================================================
#include <mutex>
#include <string>

#include "../include/xt_attn.h"

static __device__ __align__(256) float xt_ad_noalloc_scratch[XT_AD_NOALLOC_FLOATS];
static __device__ __align__(256) uint32_t xt_ad_noalloc_counters[XT_AD_NOALLOC_COUNTERS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float *g_noalloc_scratch[kMaxDevices];
uint32_t *g_noalloc_counters[kMaxDevices];
thread_local std::string g_noalloc_err;

// Device addresses of the arrays on the current device (looked up once per device). 0, or a CUDA error code.
int noalloc_setup(int dev) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_scratch[dev]) return 0;
    void *s = nullptr, *c = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&s, xt_ad_noalloc_scratch);
    if (e != cudaSuccess) return int(e);
    e = cudaGetSymbolAddress(&c, xt_ad_noalloc_counters);
    if (e != cudaSuccess) return int(e);
    e = cudaFuncSetAttribute(attn_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(AdSmem<1>::BYTES));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(AdSmem<2>::BYTES));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(AdSmem<4>::BYTES));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(AdSmem<8>::BYTES));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(AdSmem<16>::BYTES));
    if (e != cudaSuccess) return int(e);
    g_noalloc_counters[dev] = static_cast<uint32_t *>(c);
    g_noalloc_scratch[dev] = static_cast<float *>(s);
    return 0;
}

}  // namespace

extern "C" {

// q [B, Hq, 128] bf16, k_cache / v_cache [B, Hkv, L, 128] bf16, seqlens [B] int32 (device), out [B, Hq, 128] bf16;
// all device pointers on the current device. Runs the CUDA-core kernel for every group size (xt_attn_decode takes
// the tensor-core kernel for groups of 8 and 16; the two agree to rounding). Returns 0; -2 bad arguments; XT_AD_NOALLOC_TOO_BIG when the workspace would exceed the fixed array; a positive CUDA error code from
// the set-up; -1 when the launch failed.
int xt_attn_decode_noalloc(const void *q, const void *k_cache, const void *v_cache, const int32_t *seqlens, void *out,
                           int B, int Hq, int Hkv, int L, int splits, float scale, cudaStream_t stream) {
    if (!q || !k_cache || !v_cache || !seqlens || !out || B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv || L < 1 ||
        splits < 1 || splits > AD_MAX_SPLITS) {
        g_noalloc_err = "attn_decode_noalloc: bad arguments";
        return -2;
    }
    const int G = Hq / Hkv;
    if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) {
        g_noalloc_err = "attn_decode_noalloc: Hq / Hkv must be 1, 2, 4, 8 or 16";
        return -2;
    }
    const size_t units = size_t(B) * Hkv * splits * G;
    if (units * (AD_D + 2) > size_t(XT_AD_NOALLOC_FLOATS)) {
        g_noalloc_err = "attn_decode_noalloc: B * Hkv * splits * (Hq / Hkv) * 130 = " +
                        std::to_string(units * (AD_D + 2)) + " floats exceeds the fixed workspace of " +
                        std::to_string(XT_AD_NOALLOC_FLOATS) + " floats; use fewer splits or xt_attn_decode";
        return XT_AD_NOALLOC_TOO_BIG;
    }
    if (size_t(B) * Hkv > size_t(XT_AD_NOALLOC_COUNTERS)) {
        g_noalloc_err = "attn_decode_noalloc: B * Hkv exceeds the " + std::to_string(XT_AD_NOALLOC_COUNTERS) +
                        " arrival counters of the fixed workspace";
        return XT_AD_NOALLOC_TOO_BIG;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
        g_noalloc_err = "attn_decode_noalloc: no current device";
        return -2;
    }
    if (dev >= kMaxDevices) {
        g_noalloc_err = "attn_decode_noalloc: device index " + std::to_string(dev) + " exceeds the " +
                        std::to_string(kMaxDevices) + " devices of the fixed address table";
        return -2;
    }
    const int rc = noalloc_setup(dev);
    if (rc != 0) {
        g_noalloc_err = "attn_decode_noalloc: cudaGetSymbolAddress / attribute set-up failed";
        return rc;
    }
    // the counters must start at zero; everything else is written before it is read
    if (cudaMemsetAsync(g_noalloc_counters[dev], 0, sizeof(uint32_t) * size_t(B) * Hkv, stream) != cudaSuccess) {
        g_noalloc_err = "attn_decode_noalloc: clearing the counters failed";
        return -1;
    }
    AttnDecodeParams p{};
    p.q = static_cast<const __nv_bfloat16 *>(q);
    p.kc = static_cast<const __nv_bfloat16 *>(k_cache);
    p.vc = static_cast<const __nv_bfloat16 *>(v_cache);
    p.seqlens = seqlens;
    p.out = static_cast<__nv_bfloat16 *>(out);
    p.ws_o = g_noalloc_scratch[dev];
    p.ws_ml = g_noalloc_scratch[dev] + units * AD_D;
    p.counters = g_noalloc_counters[dev];
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.L = L;
    p.splits = splits;
    p.scale_log2 = scale * 1.4426950408889634f;
    dim3 grid(splits, Hkv, B);
    switch (G) {
        case 1: attn_decode_kernel<1><<<grid, AD_WARPS * 32, AdSmem<1>::BYTES, stream>>>(p); break;
        case 2: attn_decode_kernel<2><<<grid, AD_WARPS * 32, AdSmem<2>::BYTES, stream>>>(p); break;
        case 4: attn_decode_kernel<4><<<grid, AD_WARPS * 32, AdSmem<4>::BYTES, stream>>>(p); break;
        case 8: attn_decode_kernel<8><<<grid, AD_WARPS * 32, AdSmem<8>::BYTES, stream>>>(p); break;
        case 16: attn_decode_kernel<16><<<grid, AD_WARPS * 32, AdSmem<16>::BYTES, stream>>>(p); break;
        default: return -2;   // unreachable: G was checked before anything was enqueued
    }
    if (cudaGetLastError() != cudaSuccess) {
        g_noalloc_err = "attn_decode_noalloc: launch failed";
        return -1;
    }
    return 0;
}

// Text of the last error of xt_attn_decode_noalloc on this host thread.
const char *xt_attn_decode_noalloc_error(void) { return g_noalloc_err.c_str(); }

// The fixed workspace limits: out[0] = floats of the split workspace, out[1] = arrival counters.
void xt_attn_decode_noalloc_limits(long long *out) {
    out[0] = XT_AD_NOALLOC_FLOATS;
    out[1] = XT_AD_NOALLOC_COUNTERS;
}

}  // extern "C"
