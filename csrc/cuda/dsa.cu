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
#include <cudaTypedefs.h>

#include "params.h"
#include "tc_common.cuh"

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

// ------------------------------------------------------------------------------------------------ tensor-core indexer
// One CTA per (128 keys, NQ queries that share the keys' cache row): D[128 keys, 64 NQ] = K8[128, 128] . Q8^T on
// tcgen05 (kind::f8f6f4, E4M3 x E4M3, FP32 accumulation in TMEM; K = 128 = one 128-byte swizzle row), then each
// epilogue thread owns one key (one TMEM lane) and reduces its row: score[q, key] = kscale[key] *
// sum_h w[q, h] * relu(D[key, q*64 + h]) (w already carries the query's FP8 scale). Causal rows (prefill) mask keys
// past the query's position.
template <int NQ>
__global__ void __launch_bounds__(192, 1)
    dsa_index_tc_kernel(const __grid_constant__ CUtensorMap tma_k, const __grid_constant__ CUtensorMap tma_q,
                        const float *__restrict__ w, const float *__restrict__ kscale, const int64_t *__restrict__ base,
                        const int32_t *__restrict__ len, float *__restrict__ scores, int max_len, int *error) {
    constexpr int N = IDX_HEADS * NQ;
    __shared__ __align__(1024) uint8_t sk[128 * 128];
    __shared__ __align__(1024) uint8_t sq[N * 128];
    __shared__ uint64_t full, done;
    __shared__ uint32_t tmem_slot;
    __shared__ float ws[NQ][IDX_HEADS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, qg = blockIdx.y;
    const int q0 = qg * NQ;
    const int64_t row_base = base[q0];   // the NQ queries share the cache row
    int nmax = 0;
    for (int i = 0; i < NQ; ++i) nmax = max(nmax, len[q0 + i]);
    const bool any = tile * 128 < nmax;
    for (int i = threadIdx.x; i < NQ * IDX_HEADS; i += blockDim.x) ws[i / IDX_HEADS][i % IDX_HEADS] = w[size_t(q0) * IDX_HEADS + i];
    if (threadIdx.x == 0) {
        tc::mbar_init(&full, 1);
        tc::mbar_init(&done, 1);
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_slot, N < 32 ? 32 : N);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;
    if (any) {
        if (warp == 0 && lane == 0) {
            tc::mbar_arrive_expect_tx(&full, 128 * 128 + N * 128);
            tc::tma_load_2d(sk, &tma_k, &full, 0, int(row_base) + tile * 128);
            tc::tma_load_2d(sq, &tma_q, &full, 0, q0 * IDX_HEADS);
        } else if (warp == 1 && lane == 0) {
            if (tc::mbar_wait(&full, 0)) {
                tc::tc_fence_after();
                // kind::f8f6f4: D F32 (bit 4), A and B E4M3 (format 0), N / 8, M / 16
                const uint32_t idesc = (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(128 >> 4) << 24);
                const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_u32(sk)), bd = tc::sw128_kmajor_desc(tc::smem_u32(sq));
#pragma unroll
                for (int k = 0; k < 4; ++k)   // K = 32 bytes per MMA
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                 " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                                 "l"(ad + uint64_t(2 * k)), "l"(bd + uint64_t(2 * k)), "r"(idesc), "r"(k > 0 ? 1u : 0u)
                                 : "memory");
                tc::mma_commit(&done);
            } else {
                atomicExch(error, 1);
                tc::mbar_arrive(&done);   // let the epilogue go (it writes -inf)
            }
        } else if (warp >= 2) {
            const int quarter = warp & 3;
            const int key = tile * 128 + quarter * 32 + lane;
            if (lane == 0) ok = tc::mbar_wait(&done, 0);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            tc::tc_fence_after();
            const float ks = key < max_len ? kscale[row_base + key] : 0.f;
#pragma unroll
            for (int qq = 0; qq < NQ; ++qq) {
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < IDX_HEADS / 32; ++c) {
                    uint32_t r[32];
                    tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(qq * IDX_HEADS + c * 32), r);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc += ws[qq][c * 32 + i] * fmaxf(__uint_as_float(r[i]), 0.f);
                }
                if (key < max_len)
                    scores[size_t(q0 + qq) * max_len + key] = (ok && key < len[q0 + qq]) ? acc * ks : -INFINITY;
            }
        }
    } else if (threadIdx.x >= 64) {   // nothing to score in this tile: -inf for every query
        const int key = tile * 128 + threadIdx.x - 64;
        if (key < max_len)
            for (int qq = 0; qq < NQ; ++qq) scores[size_t(q0 + qq) * max_len + key] = -INFINITY;
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, N < 32 ? 32 : N);
    }
}

// ------------------------------------------------------------------------------------------------ prefill indexer
// The queries of a prefill chunk share one cache row. One CTA per (4 queries, key split): the 4 queries' FP8 Q
// [256 = 4 x 64 heads, 128] stays in shared memory, the split's 128-key tiles stream through a TMA ring, and each tile
// is one D[128 keys, 256] = K8 . Q8^T on tcgen05 (4 MMAs of K = 32 bytes) into one of two TMEM accumulators, so the
// epilogue of tile t overlaps the MMAs of tile t + 1. 576 threads:
//   warp 0      TMA producer (lane 0)
//   warp 1      TMEM owner (512 columns) and MMA issuer (lane 0)
//   warps 2-17  epilogue, one warp per (query of the group, 32-lane quarter of the accumulator): each thread owns one
//               key and reduces score[q, key] = kscale[key] * sum_h w[q, h] * relu(D[key, q * 64 + h]); keys at or
//               past the query's length get -inf up to the end of the last tile, nothing beyond it (top-k reads each
//               row only up to its length)
// Every wait is bounded; a wait that runs out sets the error word and the CTA winds down.
constexpr int IP_NQ = 4;
constexpr int IP_N = IDX_HEADS * IP_NQ;   // 256
constexpr int IP_STAGES = 6;
constexpr int IP_THREADS = 576;

struct IpSmem {
    static constexpr int Q = IP_N * 128;   // 32 KB
    static constexpr int KT = 128 * 128;   // 16 KB: a key tile
    static constexpr int BYTES = Q + IP_STAGES * KT + 1024;
};

__global__ void __launch_bounds__(IP_THREADS, 1)
    dsa_index_pf_kernel(const __grid_constant__ CUtensorMap tma_k, const __grid_constant__ CUtensorMap tma_q,
                        const float *__restrict__ w, const float *__restrict__ kscale, int64_t row_base,
                        const int32_t *__restrict__ len, float *__restrict__ scores, int Q, int max_len, int *error) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qs = smem;
    uint8_t *ring = smem + IpSmem::Q;
    __shared__ uint64_t full[IP_STAGES], empty[IP_STAGES], qfull, accf[2], acce[2];
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(16) float ws[IP_NQ][IDX_HEADS];
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.y * IP_NQ, split = blockIdx.x, splits = gridDim.x;
    int nmax = 0;
    for (int i = 0; i < IP_NQ; ++i)
        if (q0 + i < Q) nmax = max(nmax, min(len[q0 + i], max_len));
    const int ntile = (nmax + 127) / 128, per = (ntile + splits - 1) / splits;
    const int t0 = split * per, nt = min(ntile, t0 + per) - t0;
    for (int i = threadIdx.x; i < IP_NQ * IDX_HEADS; i += blockDim.x) {
        const int qi = q0 + i / IDX_HEADS;
        ws[i / IDX_HEADS][i % IDX_HEADS] = qi < Q ? w[size_t(qi) * IDX_HEADS + i % IDX_HEADS] : 0.f;
    }
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < IP_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(&qfull, 1);
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(&accf[a], 1);
            tc::mbar_init(&acce[a], 16);
        }
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tmem_slot;
    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(error, 1);
    };

    if (nt > 0) {
        if (warp == 0) {
            if (lane == 0) {
                tc::prefetch_tmap(&tma_k);
                tc::mbar_arrive_expect_tx(&qfull, IpSmem::Q);
                tc::tma_load_2d(qs, &tma_q, &qfull, 0, q0 * IDX_HEADS);
                int stage = 0;
                uint32_t phase = 0;
                for (int t = 0; t < nt && !abort_flag; ++t) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&full[stage], IpSmem::KT);
                    tc::tma_load_2d(ring + stage * IpSmem::KT, &tma_k, &full[stage], 0,
                                    int(row_base + int64_t(t0 + t) * 128));
                    if (++stage == IP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        } else if (warp == 1) {
            if (lane == 0) {
                // kind::f8f6f4: D F32 (bit 4), A and B E4M3 (format 0), N / 8, M / 16
                const uint32_t idesc = (1u << 4) | (uint32_t(IP_N >> 3) << 17) | (uint32_t(128 >> 4) << 24);
                const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_u32(qs));
                bool ok = tc::mbar_wait(&qfull, 0);
                int stage = 0;
                uint32_t phase = 0;
                for (int t = 0; t < nt && ok && !abort_flag; ++t) {
                    const int a = t & 1;
                    if (!(ok = tc::mbar_wait(&acce[a], uint32_t(((t >> 1) & 1) ^ 1)))) break;
                    if (!(ok = tc::mbar_wait(&full[stage], phase))) break;
                    tc::tc_fence_after();
                    const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_u32(ring + stage * IpSmem::KT));
#pragma unroll
                    for (int k = 0; k < 4; ++k)   // K = 32 bytes per MMA
                        asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                     " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                                         tmem + uint32_t(a * IP_N)),
                                     "l"(ad + uint64_t(2 * k)), "l"(bd + uint64_t(2 * k)), "r"(idesc),
                                     "r"(k > 0 ? 1u : 0u)
                                     : "memory");
                    tc::mma_commit(&empty[stage]);
                    tc::mma_commit(&accf[a]);
                    if (++stage == IP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) fail();
            }
        } else {
            const int qq = (warp - 2) >> 2, quarter = warp & 3;
            const int qi = q0 + qq;
            const int L = qi < Q ? min(len[qi], max_len) : 0;
            const float4 *wq = reinterpret_cast<const float4 *>(ws[qq]);
            for (int t = 0; t < nt; ++t) {
                const int a = t & 1;
                int good = 1;
                if (lane == 0) good = tc::mbar_wait(&accf[a], uint32_t((t >> 1) & 1));
                good = __shfl_sync(0xffffffffu, good, 0);
                if (!good || abort_flag) {
                    if (!good && lane == 0) fail();
                    break;
                }
                tc::tc_fence_after();
                uint32_t r[2][32];
                const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(a * IP_N + qq * IDX_HEADS);
                tc::tmem_ld32(base, r[0]);
                tc::tmem_ld32(base + 32u, r[1]);
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&acce[a]);
                const int key = (t0 + t) * 128 + quarter * 32 + lane;
                float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int h4 = 0; h4 < 8; ++h4) {
                        const float4 wv = wq[c * 8 + h4];
                        acc0 += wv.x * fmaxf(__uint_as_float(r[c][4 * h4]), 0.f);
                        acc1 += wv.y * fmaxf(__uint_as_float(r[c][4 * h4 + 1]), 0.f);
                        acc0 += wv.z * fmaxf(__uint_as_float(r[c][4 * h4 + 2]), 0.f);
                        acc1 += wv.w * fmaxf(__uint_as_float(r[c][4 * h4 + 3]), 0.f);
                    }
                if (qi < Q && key < max_len)
                    scores[size_t(qi) * max_len + key] = key < L ? (acc0 + acc1) * kscale[row_base + key] : -INFINITY;
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// Indexer queries to FP8, one warp per (query, head) row of 128: s = max(amax / 448, 1e-12), q8 = E4M3(q / s) (IEEE
// division, round to nearest even), w8 = (w * w_scale) * s, the head weight carrying the scale (relu commutes with a
// positive scale). w is BF16 [rows] (one weight per row).
__global__ void __launch_bounds__(256) dsa_quant_q_kernel(const __nv_bfloat16 *__restrict__ q,
                                                         const __nv_bfloat16 *__restrict__ w, float w_scale,
                                                         uint8_t *__restrict__ q8, float *__restrict__ w8, int rows) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint2 raw = reinterpret_cast<const uint2 *>(q + size_t(r) * IDX_DIM)[lane];
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
    float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float sc = fmaxf(m / 448.f, 1e-12f);
    const uint32_t packed = uint32_t(f32_to_e4m3(a.x / sc)) | (uint32_t(f32_to_e4m3(a.y / sc)) << 8) |
                            (uint32_t(f32_to_e4m3(b.x / sc)) << 16) | (uint32_t(f32_to_e4m3(b.y / sc)) << 24);
    reinterpret_cast<uint32_t *>(q8 + size_t(r) * IDX_DIM)[lane] = packed;
    if (lane == 0) w8[r] = (__bfloat162float(w[r]) * w_scale) * sc;
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

// Rows of stride `stride`; row r holds len[r] scores (all `stride` when len is null).
__global__ void __launch_bounds__(TK_THREADS) topk_rows_kernel(const float *__restrict__ scores, int stride, int K,
                                                               const int32_t *__restrict__ len,
                                                               int32_t *__restrict__ out) {
    __shared__ int hist[256];
    __shared__ int warp_sums[32];
    __shared__ uint32_t prefix_s;
    __shared__ int need_s, finite_s;
    const int row = blockIdx.x;
    const float *x = scores + size_t(row) * stride;
    const int n = len ? max(0, min(stride, len[row])) : stride;
    int32_t *o = out + size_t(row) * K;
    const bool vec = (stride % 4) == 0;   // rows 16-byte aligned
    // radix select of the K-th largest key among finite scores (pass 0 also counts them)
    uint32_t prefix = 0;
    int need = K;
    bool all = false;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        const uint32_t mask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
        for (int i = threadIdx.x; i < 256; i += TK_THREADS) hist[i] = 0;
        if (threadIdx.x == 0) finite_s = 0;
        __syncthreads();
        int fin = 0;
        // 4 consecutive elements per thread and step, 4 steps unrolled: 16 loads in flight per thread
#pragma unroll 4
        for (int i0 = threadIdx.x * 4; i0 < n; i0 += TK_THREADS * 4) {
            float v[4];
            if (vec && i0 + 3 < n) {
                const float4 f = *reinterpret_cast<const float4 *>(x + i0);
                v[0] = f.x;
                v[1] = f.y;
                v[2] = f.z;
                v[3] = f.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = i0 + e < n ? x[i0 + e] : -INFINITY;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (v[e] == -INFINITY) continue;
                ++fin;
                const uint32_t k = fkey(v[e]);
                if ((k & mask) == (prefix & mask)) atomicAdd(&hist[(k >> shift) & 0xFF], 1);
            }
        }
        if (pass == 0) {
            fin += __shfl_xor_sync(0xffffffffu, fin, 16);
            fin += __shfl_xor_sync(0xffffffffu, fin, 8);
            fin += __shfl_xor_sync(0xffffffffu, fin, 4);
            fin += __shfl_xor_sync(0xffffffffu, fin, 2);
            fin += __shfl_xor_sync(0xffffffffu, fin, 1);
            if ((threadIdx.x & 31) == 0) atomicAdd(&finite_s, fin);
        }
        __syncthreads();
        if (pass == 0 && finite_s <= K) {
            all = true;
            break;
        }
        if (threadIdx.x < 32) {   // bucket of the need-th largest: lane l sums buckets 255-8l .. 248-8l, warp scan
            const int l = threadIdx.x;
            int c8 = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) c8 += hist[255 - 8 * l - j];
            int inc = c8;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (l >= o) inc += y;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, inc >= need);
            const int L = hit ? __ffs(hit) - 1 : 31;
            if (l == L) {
                int acc = inc - c8, b = 255 - 8 * l;
                for (int j = 0; j < 7; ++j, --b) {
                    if (acc + hist[b] >= need) break;
                    acc += hist[b];
                }
                prefix_s = prefix | (uint32_t(b) << shift);
                need_s = need - acc;
            }
        }
        __syncthreads();
        prefix = prefix_s;
        need = need_s;
        __syncthreads();
    }
    // ordered compaction, 4 consecutive elements per thread and one block scan per chunk: keys above the threshold,
    // then `need` of the keys equal to it, in index order
    const uint32_t thr = prefix;
    int gt_before = 0, eq_before = 0;
    for (int c0 = 0; c0 < n; c0 += TK_THREADS * 4) {
        const int i0 = c0 + threadIdx.x * 4;
        int gt[4], eq[4], cg = 0, ce = 0;
        float vv[4];
        if (vec && i0 + 3 < n) {
            const float4 f = *reinterpret_cast<const float4 *>(x + i0);
            vv[0] = f.x;
            vv[1] = f.y;
            vv[2] = f.z;
            vv[3] = f.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) vv[e] = i0 + e < n ? x[i0 + e] : -INFINITY;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float v = vv[e];
            const bool fin = v > -INFINITY;
            const uint32_t k = fin ? fkey(v) : 0u;
            gt[e] = all ? int(fin) : int(fin && k > thr);
            eq[e] = all ? 0 : int(fin && k == thr);
            cg += gt[e];
            ce += eq[e];
        }
        int tot;
        const int pre = block_scan((cg << 16) | ce, warp_sums, &tot);
        int pg = gt_before + (pre >> 16), pe = eq_before + (pre & 0xFFFF);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int pos = pg + min(pe, need);
            if ((gt[e] || (eq[e] && pe < need)) && pos < K) o[pos] = i0 + e;
            pg += gt[e];
            pe += eq[e];
        }
        gt_before += tot >> 16;
        eq_before += tot & 0xFFFF;
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

namespace {
bool dsa_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult qr;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    cuuint64_t dims[2] = {cuuint64_t(IDX_DIM), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(IDX_DIM)};
    cuuint32_t box[2] = {cuuint32_t(IDX_DIM), box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

// Tensor-core indexer: q8 [Q, 64, 128] E4M3 (queries pre-quantized, w carries their scales), codes [slots, 128] E4M3,
// nq queries per CTA share a cache row (1 for decode rows, 2 for a prefill chunk of one sequence).
int xt_dsa_index_tc(const void *q8, const float *w, const void *codes, int64_t slots, const float *kscale,
                    const int64_t *base, const int32_t *len, float *scores, int Q, int max_len, int nq, int *error,
                    cudaStream_t stream) {
    if (Q <= 0 || max_len <= 0 || (nq != 1 && nq != 2) || Q % nq) return -2;
    CUtensorMap mk, mq;
    if (!dsa_map(&mk, codes, uint64_t(slots), 128) || !dsa_map(&mq, q8, uint64_t(Q) * IDX_HEADS, IDX_HEADS * nq))
        return -3;
    dim3 grid((max_len + 127) / 128, Q / nq);
    if (nq == 1)
        dsa_index_tc_kernel<1><<<grid, 192, 0, stream>>>(mk, mq, w, kscale, base, len, scores, max_len, error);
    else
        dsa_index_tc_kernel<2><<<grid, 192, 0, stream>>>(mk, mq, w, kscale, base, len, scores, max_len, error);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Prefill indexer: the Q queries share the cache row starting at slot row_base; query i scores keys
// [0, len[i]) of it (scores [Q, max_len], -inf from len[i] to the end of its last key tile). splits key ranges per
// group of 4 queries (0: chosen here).
int xt_dsa_index_pf(const void *q8, const float *w, const void *codes, int64_t slots, const float *kscale,
                    int64_t row_base, const int32_t *len, float *scores, int Q, int max_len, int splits, int *error,
                    cudaStream_t stream) {
    if (Q <= 0 || max_len <= 0 || splits < 0) return -2;
    CUtensorMap mk, mq;
    if (!dsa_map(&mk, codes, uint64_t(slots), 128) || !dsa_map(&mq, q8, uint64_t(Q) * IDX_HEADS, IP_N)) return -3;
    const int groups = (Q + IP_NQ - 1) / IP_NQ;
    if (groups > 65535) return -2;
    if (splits == 0) {   // about four CTAs per SM over the chunk, at least 8 key tiles per CTA
        int sms = 148, dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int tiles = (max_len + 127) / 128;
        splits = max(1, min((4 * sms + groups - 1) / groups, tiles / 8));
    }
    if (xt_smem_optin(dsa_index_pf_kernel, IpSmem::BYTES) != cudaSuccess) return -4;
    dsa_index_pf_kernel<<<dim3(splits, groups), IP_THREADS, IpSmem::BYTES, stream>>>(mk, mq, w, kscale, row_base, len,
                                                                                  scores, Q, max_len, error);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_dsa_quant_q(const void *q, const void *w, float w_scale, void *q8, float *w8, int rows, cudaStream_t stream) {
    if (rows <= 0) return 0;
    dsa_quant_q_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(q),
                                                          static_cast<const __nv_bfloat16 *>(w), w_scale,
                                                          static_cast<uint8_t *>(q8), w8, rows);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_topk_rows(const float *scores, int rows, int n, int K, const int32_t *len, int32_t *out, cudaStream_t stream) {
    if (rows <= 0 || n <= 0 || K <= 0) return -2;
    topk_rows_kernel<<<rows, TK_THREADS, 0, stream>>>(scores, n, K, len, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
