// Skinny BF16 GEMM for decode-sized inputs on the 5th-generation tensor cores: y[M, N] = x[M, K] . W[N, K]^T (+ add),
// M <= 32 tokens (a decode step's projections, LM head).
//
// With a handful of token rows every weight byte feeds at most 32 multiply-adds, so a CUDA-core GEMV runs out of FP32
// issue slots long before HBM bandwidth at 8 or more rows. Here the weights are the MMA's M operand (swap-AB): a CTA
// owns 128 weight rows and a range of K, streams [128 x 64] weight tiles and the matching [MP x 64] token tile
// (MP = 16 or 32, rows past M zero-filled by TMA) through a 6-stage TMA ring (two CTAs per SM, so one CTA's epilogue
// overlaps the other's stream), and accumulates D[128, MP] = W . X^T in TMEM with tcgen05 (kind::f16, 128 x MP x 16
// per instruction). 192 threads:
//   warp 0      TMA producer (lane 0): the first stages' weight tiles are requested before the programmatic-dependent-
//               launch wait (weights do not depend on the previous kernel), the token tiles after it
//   warp 1      TMEM owner (32 columns) and MMA issuer (lane 0)
//   warps 2-5   epilogue, one weight row per thread: its MP accumulators -> y (BF16, + add) or, when K is split over
//               several CTAs, FP32 partials [split, M, N] that skinny_reduce sums in split order (deterministic)
// Every wait is bounded; a wait that runs out sets the error word and the CTA winds down.
#include <cudaTypedefs.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int SK_BN = 128, SK_BK = 64, SK_STAGES = 6, SK_THREADS = 192;   // two CTAs per SM

template <int MP>
struct SkSmem {
    static constexpr int W = SK_BN * SK_BK * 2;   // 16 KB
    static constexpr int X = MP * SK_BK * 2;      // 2 or 4 KB (a multiple of 1024: every tile 1024-aligned)
    static constexpr int STAGE = W + X;
    static constexpr int BYTES = SK_STAGES * STAGE + 1024;
};

template <int MP>
__global__ void __launch_bounds__(SK_THREADS)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                       const __nv_bfloat16 *__restrict__ add, __nv_bfloat16 *__restrict__ y, float *__restrict__ part,
                       int M, int N, int kb_per, int nkb_total, int *error) {
    using S = SkSmem<MP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[SK_STAGES], empty[SK_STAGES], done;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * SK_BN, split = blockIdx.y;
    const int kb0 = split * kb_per, nkb = min(nkb_total - kb0, kb_per);
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < SK_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(&done, 1);
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_slot, 32);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0 && nkb > 0) {
            tc::prefetch_tmap(&tma_w);
            tc::prefetch_tmap(&tma_x);
            const int pre = min(nkb, SK_STAGES);
            for (int i = 0; i < pre; ++i) {   // weights first: they do not depend on the previous kernel
                tc::mbar_arrive_expect_tx(&full[i], S::STAGE);
                tc::tma_load_2d(smem + i * S::STAGE, &tma_w, &full[i], (kb0 + i) * SK_BK, n0);
            }
            pdl_wait();
            for (int i = 0; i < pre; ++i)
                tc::tma_load_2d(smem + i * S::STAGE + S::W, &tma_x, &full[i], (kb0 + i) * SK_BK, 0);
            int stage = 0;
            uint32_t phase = 1;   // the ring's second pass
            for (int i = pre; i < nkb && !abort_flag; ++i) {
                if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                    abort_flag = 1;
                    atomicExch(error, 1);
                    break;
                }
                tc::mbar_arrive_expect_tx(&full[stage], S::STAGE);
                tc::tma_load_2d(smem + stage * S::STAGE, &tma_w, &full[stage], (kb0 + i) * SK_BK, n0);
                tc::tma_load_2d(smem + stage * S::STAGE + S::W, &tma_x, &full[stage], (kb0 + i) * SK_BK, 0);
                if (++stage == SK_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16_f32(SK_BN, MP);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int i = 0; i < nkb && !abort_flag; ++i) {
                if (!(ok = tc::mbar_wait(&full[stage], phase))) break;
                tc::tc_fence_after();
                const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_u32(smem + stage * S::STAGE));
                const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_u32(smem + stage * S::STAGE + S::W));
#pragma unroll
                for (int k = 0; k < SK_BK / 16; ++k)
                    tc::mma_f16(tmem, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc, (i > 0 || k > 0) ? 1u : 0u);
                tc::mma_commit(&empty[stage]);
                if (++stage == SK_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) {
                abort_flag = 1;
                atomicExch(error, 1);
            }
            if (ok && nkb > 0) tc::mma_commit(&done);
            else tc::mbar_arrive(&done);   // let the epilogue go
        }
    } else {
        pdl_wait();
        const int quarter = warp & 3;
        const int n = n0 + quarter * 32 + lane;
        int good = 1;
        if (lane == 0) good = tc::mbar_wait(&done, 0);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good && lane == 0) atomicExch(error, 1);
        tc::tc_fence_after();
        uint32_t r[32];
        tc::tmem_ld32(tmem + (uint32_t(quarter * 32) << 16), r);
        tc::tmem_ld_wait();
        if (good && !abort_flag && nkb > 0 && n < N) {
            if (part) {
                float *dst = part + size_t(split) * M * N + n;
#pragma unroll
                for (int m = 0; m < MP; ++m)
                    if (m < M) dst[size_t(m) * N] = __uint_as_float(r[m]);
            } else {
#pragma unroll
                for (int m = 0; m < MP; ++m)
                    if (m < M) {
                        float v = __uint_as_float(r[m]);
                        if (add) v += __bfloat162float(add[size_t(m) * N + n]);
                        y[size_t(m) * N + n] = __float2bfloat16(v);
                    }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 32);
    }
}

// y[m, n] = sum over splits s (in order) of part[s, m, n] (+ add), four columns per thread
__global__ void __launch_bounds__(256) skinny_reduce_kernel(const float *__restrict__ part, int splits, int M, int N,
                                                           const __nv_bfloat16 *__restrict__ add,
                                                           __nv_bfloat16 *__restrict__ y) {
    pdl_wait();
    pdl_trigger();
    const long long i = (blockIdx.x * 256ll + threadIdx.x) * 4;
    const long long total = (long long)M * N;
    if (i >= total) return;
    const size_t plane = size_t(M) * N;
    if (i + 3 < total && N % 4 == 0) {
        float4 acc = reinterpret_cast<const float4 *>(part + i)[0];
        for (int s = 1; s < splits; ++s) {
            const float4 v = reinterpret_cast<const float4 *>(part + s * plane + i)[0];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (add) {
            const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(add + i);
            const float2 p = __bfloat1622float2(a2[0]), q = __bfloat1622float2(a2[1]);
            acc.x += p.x;
            acc.y += p.y;
            acc.z += q.x;
            acc.w += q.y;
        }
        __nv_bfloat162 o[2] = {__floats2bfloat162_rn(acc.x, acc.y), __floats2bfloat162_rn(acc.z, acc.w)};
        *reinterpret_cast<uint2 *>(y + i) = *reinterpret_cast<uint2 *>(o);
    } else {
        for (long long e = i; e < total && e < i + 4; ++e) {
            float acc = 0.f;
            for (int s = 0; s < splits; ++s) acc += part[s * plane + e];
            if (add) acc += __bfloat162float(add[e]);
            y[e] = __float2bfloat16(acc);
        }
    }
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 sk_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult qr;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

bool sk_map(CUtensorMap *map, const void *ptr, int rows, int K, int box_rows) {
    auto fn = sk_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    cuuint32_t box[2] = {SK_BK, cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

}  // namespace xt

using namespace xt;

extern "C" {

// The number of K splits skinny_gemm uses for (N, K): about two CTAs per SM, at least 4 k-blocks of 64 per CTA.
int xt_skinny_splits(int N, int K, int sms) {
    const int nblk = (N + SK_BN - 1) / SK_BN, nkb = K / SK_BK;
    const int want = (2 * sms + nblk - 1) / nblk;
    return std::max(1, std::min(want, nkb / 4));
}

// y [M, N] BF16 = x [M, K] . W [N, K]^T (+ add [M, N]); M <= 32, K % 64 == 0, rows 16-byte aligned. splits > 1
// needs part (FP32 [splits, M, N]).
int xt_skinny_gemm(const void *x, const void *W, const void *add, void *y, float *part, int M, int N, int K,
                   int splits, int *error, cudaStream_t stream) {
    if (M < 1 || M > 32 || N < 1 || K < SK_BK || K % SK_BK || splits < 1) return -2;
    if (splits > 1 && !part) return -2;
    const int nkb = K / SK_BK, kb_per = (nkb + splits - 1) / splits;
    splits = (nkb + kb_per - 1) / kb_per;
    const int MP = M <= 16 ? 16 : 32;
    CUtensorMap mw, mx;
    if (!sk_map(&mw, W, N, K, SK_BN) || !sk_map(&mx, x, M, K, MP)) return -3;
    const dim3 grid((N + SK_BN - 1) / SK_BN, splits);
    float *p = splits > 1 ? part : nullptr;
    auto A = static_cast<const __nv_bfloat16 *>(add);
    auto Y = static_cast<__nv_bfloat16 *>(y);
    cudaError_t e;
    if (MP == 16) {
        if (xt_smem_optin(skinny_gemm_kernel<16>, SkSmem<16>::BYTES) != cudaSuccess) return -4;
        e = xt_launch(skinny_gemm_kernel<16>, grid, dim3(SK_THREADS), size_t(SkSmem<16>::BYTES), stream, mw, mx,
                      p ? nullptr : A, Y, p, M, N, kb_per, nkb, error);
    } else {
        if (xt_smem_optin(skinny_gemm_kernel<32>, SkSmem<32>::BYTES) != cudaSuccess) return -4;
        e = xt_launch(skinny_gemm_kernel<32>, grid, dim3(SK_THREADS), size_t(SkSmem<32>::BYTES), stream, mw, mx,
                      p ? nullptr : A, Y, p, M, N, kb_per, nkb, error);
    }
    if (e != cudaSuccess) return -1;
    if (p) {
        const long long quads = ((long long)M * N + 3) / 4;
        e = xt_launch(skinny_reduce_kernel, dim3(unsigned((quads + 255) / 256)), dim3(256), 0, stream,
                      static_cast<const float *>(p), splits, M, N, A, Y);
        if (e != cudaSuccess) return -1;
    }
    return 0;
}

}  // extern "C"
