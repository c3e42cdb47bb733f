// Persistent warp-specialized BF16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a:
//   D[M, N] (bf16) = A[M, K] . B[N, K]^T (+ R[M, N]),   A and B K-major (a torch x @ W^T), FP32 accumulation.
//
// One CTA per SM (grid = min(tiles, SMs)), 6 warps:
//   warp 0    TMA producer: A and B k-blocks (64 elements = one 128-byte swizzle row) into a 4-stage ring
//   warp 1    TMEM owner and MMA issuer: one elected thread issues 4 tcgen05.mma (K = 16 each) per k-block into the
//             tile's accumulator; tcgen05.commit frees the ring stage when they complete, and signals the epilogue
//             after the tile's last k-block
//   warps 2-5 epilogue: tcgen05.ld of 32 columns at a time from the warp's 32 TMEM lanes (= tile rows), BF16 store
// The accumulator is double buffered in TMEM (2 x BN columns), so the epilogue of tile i overlaps the mainloop of
// tile i+1. Tiles are walked column panel by column panel, so CTAs running at the same time share B in L2.
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA winds down (the producer
// first waits, again bounded, for the loads it issued) and frees its TMEM.
#include <cudaTypedefs.h>
#include <stdlib.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int TC_BM = 128, TC_BK = 64, TC_STAGES = 4, TC_THREADS = 192;
constexpr int TC_GROUP_M = 16;   // 128-row tiles per raster group (CTA-pair kernel: 8 of 256 rows)

// 32 FP32 accumulator columns of one output row -> BF16 (+ residual), 16-byte stores where the row allows
XT_DEV void store_row32(__nv_bfloat16 *D, const __nv_bfloat16 *R, const uint32_t (&r)[32], int row, int col, int N) {
    __nv_bfloat16 *dst = D + size_t(row) * N + col;
    const __nv_bfloat16 *res = R ? R + size_t(row) * N + col : nullptr;
    if (col + 32 <= N && (N % 8) == 0) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(r[v * 8 + i]);
            if (res) {
                uint4 rv = *reinterpret_cast<const uint4 *>(res + v * 8);
                const __nv_bfloat162 *r2 = reinterpret_cast<const __nv_bfloat162 *>(&rv);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 g = __bfloat1622float2(r2[i]);
                    f[2 * i] += g.x;
                    f[2 * i + 1] += g.y;
                }
            }
            uint4 o;
            __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            *reinterpret_cast<uint4 *>(dst + v * 8) = o;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {   // static indices keep r in registers
            if (col + i < N) {
                float f = __uint_as_float(r[i]);
                if (res) f += __bfloat162float(res[i]);
                dst[i] = __float2bfloat16(f);
            }
        }
    }
}

template <int BN>
struct TcSmem {
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;
    static constexpr int B_BYTES = BN * TC_BK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int BYTES = TC_STAGES * STAGE + 1024 /*barriers*/ + 1024 /*alignment*/;
};

// 32 FP32 accumulator columns of one output row stored as FP32 (the router logits of a prefill call)
XT_DEV void store_row32_f32(float *D, const uint32_t (&r)[32], int row, int col, int N) {
    float *dst = D + size_t(row) * N + col;
    if (col + 32 <= N && (N % 4) == 0) {
#pragma unroll
        for (int v = 0; v < 8; ++v)
            reinterpret_cast<float4 *>(dst)[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                             __uint_as_float(r[4 * v + 2]),
                                                             __uint_as_float(r[4 * v + 3]));
    } else {
        for (int i = 0; i < 32 && col + i < N; ++i) dst[i] = __uint_as_float(r[i]);
    }
}

template <int BN, bool F32 = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   __nv_bfloat16 *__restrict__ D, const __nv_bfloat16 *__restrict__ R, int M, int N, int K,
                   int *error) {
    using L = TcSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + TC_STAGES * L::STAGE);
    uint64_t *empty = full + TC_STAGES;
    uint64_t *tfull = empty + TC_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (M + TC_BM - 1) / TC_BM, tiles_n = (N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n, kblocks = (K + TC_BK - 1) / TC_BK;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < TC_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 4);   // one arrival per epilogue warp
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_a);
        tc::prefetch_tmap(&tma_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 2 * BN);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;   // loads issued and not yet known complete (for the wind-down)
            for (int tile = blockIdx.x; tile < tiles && !abort_flag; tile += gridDim.x) {
                int tm, tn;
                tc::tile_coords(tile, tiles_m, tiles_n, TC_GROUP_M, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *sa = smem + stage * L::STAGE;
                    uint8_t *sb = sa + L::A_BYTES;
                    tc::mbar_arrive_expect_tx(&full[stage], L::STAGE);
                    tc::tma_load_2d(sa, &tma_a, &full[stage], kb * TC_BK, tm * TC_BM);
                    tc::tma_load_2d(sb, &tma_b, &full[stage], kb * TC_BK, tn * BN);
                    issued = min(issued + 1, TC_STAGES);
                    if (++stage == TC_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (abort_flag) {   // let the loads in flight land before the CTA goes away
                for (int i = 0; i < issued; ++i) {
                    if (--stage < 0) {
                        stage = TC_STAGES - 1;
                        phase ^= 1;
                    }
                    tc::mbar_wait(&full[stage], phase, 1u << 20);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16_f32(TC_BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = blockIdx.x; tile < tiles && !abort_flag; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t use = uint32_t(local >> 1);
                if (!tc::mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * L::STAGE);
                    const uint32_t sb = sa + L::A_BYTES;
                    const uint64_t adesc = tc::sw128_kmajor_desc(sa), bdesc = tc::sw128_kmajor_desc(sb);
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; ++k)   // K = 16 per MMA: 32 bytes further in the swizzle atom
                        tc::mma_f16(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                    (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&empty[stage]);
                    if (++stage == TC_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit(&tfull[acc]);
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, i.e. tile rows
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int local = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            int tm, tn;
                tc::tile_coords(tile, tiles_m, tiles_n, TC_GROUP_M, tm, tn);
            const int acc = local & 1;
            const uint32_t use = uint32_t(local >> 1);
            bool ok = true;
            if (lane == 0) ok = tc::mbar_wait(&tfull[acc], use & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_flag) {
                if (lane == 0) fail();
                break;
            }
            __syncwarp();
            tc::tc_fence_after();
            const int row = tm * TC_BM + row_in_tile;
            const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32(base + uint32_t(c0), r);
                tc::tmem_ld_wait();
                const int col = tn * BN + c0;
                if (row < M && col < N) {
                    if constexpr (F32)
                        store_row32_f32(reinterpret_cast<float *>(D), r, row, col, N);
                    else
                        store_row32(D, R, r, row, col, N);
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * BN);
    }
}

// ------------------------------------------------------------------------------------------------ CTA-pair variant
// Same warp roles, on a cluster of two CTAs (two SMs) sharing 256 x BN tiles through tcgen05 cta_group::2: each CTA
// loads its 128 rows of A and its BN/2 rows of B per k-block (half the B traffic per SM of the single-CTA kernel), the
// leader (even CTA) issues the MMAs for both, and each CTA's epilogue drains its own 128 accumulator rows. Barriers:
// full[s] lives in the leader and counts the bytes of both CTAs' loads; empty[s] and tfull[b] live in each CTA and
// are signalled by the leader's commits (one per CTA); tempty[b] lives in the leader and counts the 8 epilogue warps.
constexpr int TC2_STAGES = 6;

template <int BN>
struct Tc2Smem {
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;          // this CTA's 128 rows
    static constexpr int B_BYTES = (BN / 2) * TC_BK * 2;        // this CTA's BN/2 rows
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int BYTES = TC2_STAGES * STAGE + 1024 + 1024;
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    __nv_bfloat16 *__restrict__ D, const __nv_bfloat16 *__restrict__ R, int M, int N, int K,
                    int *error) {
    using L = Tc2Smem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + TC2_STAGES * L::STAGE);
    uint64_t *empty = full + TC2_STAGES;
    uint64_t *tfull = empty + TC2_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int tiles_m = (M + 2 * TC_BM - 1) / (2 * TC_BM), tiles_n = (N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n, kblocks = (K + TC_BK - 1) / TC_BK;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < TC2_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 8);   // the epilogue warps of both CTAs
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_a);
        tc::prefetch_tmap(&tma_b);
    }
    if (warp == 1) {
        tc::tmem_alloc_pair(tmem_slot, 2 * BN);
        tc::tmem_relinquish_pair();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();   // both CTAs' barriers exist before any remote arrive or load completes on them
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = pair; tile < tiles && !abort_flag; tile += pairs) {
                int tm, tn;
                tc::tile_coords(tile, tiles_m, tiles_n, TC_GROUP_M / 2, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *sa = smem + stage * L::STAGE;
                    uint8_t *sb = sa + L::A_BYTES;
                    if (leader) tc::mbar_arrive_expect_tx(&full[stage], 2 * L::STAGE);
                    tc::tma_load_2d_pair(sa, &tma_a, &full[stage], kb * TC_BK, tm * 2 * TC_BM + int(rank) * TC_BM);
                    tc::tma_load_2d_pair(sb, &tma_b, &full[stage], kb * TC_BK, tn * BN + int(rank) * (BN / 2));
                    if (++stage == TC2_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = tc::idesc_bf16_f32(2 * TC_BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = pair; tile < tiles && !abort_flag; tile += pairs, ++local) {
                const int acc = local & 1;
                const uint32_t use = uint32_t(local >> 1);
                if (!tc::mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * L::STAGE);
                    const uint32_t sb = sa + L::A_BYTES;
                    const uint64_t adesc = tc::sw128_kmajor_desc(sa), bdesc = tc::sw128_kmajor_desc(sb);
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; ++k)
                        tc::mma_f16_pair(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                         (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit_pair(tc::mapa(&empty[stage], 0));
                    tc::mma_commit_pair(tc::mapa(&empty[stage], 1));
                    if (++stage == TC2_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit_pair(tc::mapa(&tfull[acc], 0));
                tc::mma_commit_pair(tc::mapa(&tfull[acc], 1));
            }
        }
    } else {
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int local = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++local) {
            int tm, tn;
                tc::tile_coords(tile, tiles_m, tiles_n, TC_GROUP_M / 2, tm, tn);
            const int acc = local & 1;
            const uint32_t use = uint32_t(local >> 1);
            bool ok = true;
            if (lane == 0) ok = tc::mbar_wait(&tfull[acc], use & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_flag) {
                if (lane == 0) fail();
                break;
            }
            __syncwarp();
            tc::tc_fence_after();
            const int row = tm * 2 * TC_BM + int(rank) * TC_BM + row_in_tile;
            const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32(base + uint32_t(c0), r);
                tc::tmem_ld_wait();
                const int col = tn * BN + c0;
                if (row < M && col < N) store_row32(D, R, r, row, col, N);
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_cluster(tc::mapa(&tempty[acc], 0));
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::cluster_sync();   // no CTA leaves while its pair may still signal its barriers
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc_pair(tmem, 2 * BN);
    }
}

}  // namespace xt

using namespace xt;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [rows, cols] row-major BF16, box = box_rows x 64 columns, 128-byte swizzle
bool make_map(CUtensorMap *map, const void *ptr, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
    cuuint32_t box[2] = {cuuint32_t(TC_BK), cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

template <int BN, bool F32 = false>
int launch(const void *A, const void *B, void *Dp, const void *R, int M, int N, int K, int *error,
           cudaStream_t stream) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, A, M, K, TC_BM) || !make_map(&mb, B, N, K, BN)) return -3;
    const int smem = TcSmem<BN>::BYTES;
    if (xt_smem_optin(gemm_tc_kernel<BN, F32>, smem) != cudaSuccess) return -4;
    const int tiles = ((M + TC_BM - 1) / TC_BM) * ((N + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gemm_tc_kernel<BN, F32><<<grid, TC_THREADS, smem, stream>>>(ma, mb, static_cast<__nv_bfloat16 *>(Dp),
                                                                static_cast<const __nv_bfloat16 *>(R), M, N, K, error);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <int BN>
int launch_pair(const void *A, const void *B, void *Dp, const void *R, int M, int N, int K, int *error,
                cudaStream_t stream) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, A, M, K, TC_BM) || !make_map(&mb, B, N, K, BN / 2)) return -3;
    const int smem = Tc2Smem<BN>::BYTES;
    if (xt_smem_optin(gemm_tc2_kernel<BN>, smem) != cudaSuccess) return -4;
    const int tiles = ((M + 2 * TC_BM - 1) / (2 * TC_BM)) * ((N + BN - 1) / BN);
    int pairs = num_sms() / 2;
    if (tiles < pairs) pairs = tiles;
    gemm_tc2_kernel<BN><<<2 * pairs, TC_THREADS, smem, stream>>>(ma, mb, static_cast<__nv_bfloat16 *>(Dp),
                                                                 static_cast<const __nv_bfloat16 *>(R), M, N, K,
                                                                 error);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

extern "C" int xt_gemm_tc(const void *A, const void *B, void *D, const void *R, int M, int N, int K, int *error,
                          cudaStream_t stream) {
    // TMA: row strides must be multiples of 16 bytes; the k coordinates are multiples of 64 elements
    if (M <= 0 || N <= 0 || K <= 0 || K % 8 || !error) return -2;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return -2;
    static const int mode = [] {   // XTIER_GEMM_PAIR=1 selects the CTA-pair kernel (measured on par, not faster)
        const char *v = getenv("XTIER_GEMM_PAIR");
        return v ? atoi(v) : 0;
    }();
    // the CTA-pair kernel once there are enough 256-row tiles to fill the SM pairs
    if (mode && M >= 1024 && N >= 256 && N % 16 == 0) {
        if (N >= 2048) return launch_pair<256>(A, B, D, R, M, N, K, error, stream);
        return launch_pair<128>(A, B, D, R, M, N, K, error, stream);
    }
    if (N >= 2048) return launch<256>(A, B, D, R, M, N, K, error, stream);
    return launch<128>(A, B, D, R, M, N, K, error, stream);
}

// D[M, N] FP32 = A[M, K] . B[N, K]^T (BF16 operands): prefill router logits, kept in FP32 like the decode router's.
extern "C" int xt_gemm_tc_f32(const void *A, const void *B, float *D, int M, int N, int K, int *error,
                              cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || K % 8 || !error) return -2;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return -2;
    return launch<128, true>(A, B, D, nullptr, M, N, K, error, stream);
}
