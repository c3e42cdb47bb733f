// Tensor-parallel GEMMs fused with their collective over NVLink peer memory (sm_100a, tcgen05 + TMEM + TMA):
//
//   MODE_RS  GEMM -> reduce-scatter:  rank r holds A_r [M, K_r], B_r [N, K_r] (a row-parallel layer: K split over the
//            ranks); the full result D = sum_r A_r B_r^T is reduce-scattered by rows (rank j owns rows
//            [j*M/W, (j+1)*M/W)). The epilogue stores every output tile as a BF16 partial straight into its owner's
//            receive slot [src][rows][N] over NVLink and then releases a per-(src, tile) flag; the tile walk starts
//            with the next rank's rows, so the transfers of finished tiles overlap the MMAs of the next ones; the
//            rank's own tiles come last, and their epilogue waits for the peers' partials of the same tile and sums
//            the W partials in rank order (FP32, + residual) into the output rows: no separate reduction pass.
//   MODE_AG  all-gather -> GEMM:      rank r holds the row shard A_r [M/W, K] (a column-parallel layer: B_r [N_r, K]);
//            two push warps of every CTA store A_r into every peer's gather buffer [M, K] in 128-row blocks, each
//            released with a flag, while the same kernel's MMAs run: the walk starts with the local rows, which the
//            TMA producer reads straight from A_r; a peer's block is loaded (from this rank's own gather buffer)
//            once its flag has arrived (bounded wait).
// TMA only ever reads this rank's own memory; peer memory is touched only with plain stores and flag loads.
// The receive and gather regions are double buffered by call parity (a rank can run at most one call ahead of its
// peers), and a per-call epoch in device memory tags the flags, so the calls replay from CUDA graphs with no host
// work. Every wait is bounded; a wait that runs out sets the error word.
#include <cudaTypedefs.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {


constexpr int TP_BM = 128, TP_BK = 64, TP_STAGES = 4, TP_THREADS = 192, TP_THREADS_AG = 256;
constexpr int TP_GROUP_M = 16;   // raster groups of 128-row tiles (L2 reuse of A and B)

template <int BN>
struct TpSmem {
    static constexpr int A_BYTES = TP_BM * TP_BK * 2;
    static constexpr int B_BYTES = BN * TP_BK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int BYTES = TP_STAGES * STAGE + 1024 + 1024;
};

XT_DEV bool tp_wait_flag(const volatile uint32_t *f, uint32_t epoch, unsigned long long timeout_ns) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) != epoch)
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    return true;
}

template <int BN, int MODE>
__global__ void __launch_bounds__(TP_THREADS_AG, 1)
    gemm_tp_kernel(const __grid_constant__ CUtensorMap tma_a0, const __grid_constant__ CUtensorMap tma_a1,
                   const __grid_constant__ CUtensorMap tma_b, const __grid_constant__ CUtensorMap tma_l, TpParams p) {
    using L = TpSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + TP_STAGES * L::STAGE);
    uint64_t *empty = full + TP_STAGES;
    uint64_t *tfull = empty + TP_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int Mo = p.M / p.W;                       // rows per rank
    const int mb_per_owner = Mo / TP_BM;            // 128-row blocks per rank
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tpo = mb_per_owner * tiles_n;         // tiles per owner
    const int tiles = tpo * p.W, kblocks = (p.K + TP_BK - 1) / TP_BK;
    const uint32_t epoch = p.state[0] + 1;
    const int par = epoch & 1;
    // walk index -> (owner, tile row, tile column); RS starts with the next rank, AG with this rank
    auto tile_at = [&](int i, int &owner, int &tm, int &tn, int &j) {
        owner = (p.rank + (MODE == 0 ? 1 : 0) + i / tpo) % p.W;
        j = i % tpo;
        int tml;
        tc::tile_coords(j, mb_per_owner, tiles_n, TP_GROUP_M, tml, tn);
        tm = owner * mb_per_owner + tml;
    };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < TP_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 4);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(par ? &tma_a1 : &tma_a0);
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
    const CUtensorMap *tma_a = par ? &tma_a1 : &tma_a0;   // AG: the gather region of this call's parity
    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(p.error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            const uint8_t *me = reinterpret_cast<const uint8_t *>(p.peer[p.rank]);
            for (int i = blockIdx.x; i < tiles && !abort_flag; i += gridDim.x) {
                int owner, tm, tn, j;
                tile_at(i, owner, tm, tn, j);
                const bool local_rows = MODE == 1 && owner == p.rank;   // AG: this rank's rows come from a_shard
                if (MODE == 1 && !local_rows) {   // a peer's A block must have landed in this rank's gather buffer
                    const volatile uint32_t *f =
                        reinterpret_cast<const volatile uint32_t *>(me + (par ? p.off_flags[1] : p.off_flags[0])) + tm;
                    if (!tp_wait_flag(f, epoch, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    asm volatile("fence.proxy.async.global;\n" ::: "memory");   // generic-proxy writes -> TMA reads
                }
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *sa = smem + stage * L::STAGE;
                    uint8_t *sb = sa + L::A_BYTES;
                    tc::mbar_arrive_expect_tx(&full[stage], L::STAGE);
                    if (local_rows)
                        tc::tma_load_2d(sa, &tma_l, &full[stage], kb * TP_BK, (tm - owner * mb_per_owner) * TP_BM);
                    else
                        tc::tma_load_2d(sa, tma_a, &full[stage], kb * TP_BK, tm * TP_BM);
                    tc::tma_load_2d(sb, &tma_b, &full[stage], kb * TP_BK, tn * BN);
                    issued = min(issued + 1, TP_STAGES);
                    if (++stage == TP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (abort_flag) {
                for (int q = 0; q < issued; ++q) {
                    if (--stage < 0) {
                        stage = TP_STAGES - 1;
                        phase ^= 1;
                    }
                    tc::mbar_wait(&full[stage], phase, 1u << 20);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16_f32(TP_BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int i = blockIdx.x; i < tiles && !abort_flag; i += gridDim.x, ++local) {
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
                    for (int k = 0; k < TP_BK / 16; ++k)
                        tc::mma_f16(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                    (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&empty[stage]);
                    if (++stage == TP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit(&tfull[acc]);
            }
        }
    } else if (warp >= 6) {
        // AG push warps (MODE 1 only): this rank's 128-row blocks into every peer's gather buffer over NVLink, each
        // released with a flag; the blocks are spread over the CTAs, and the GEMM's local tiles run meanwhile
        if (MODE == 1) {
            const int pt = threadIdx.x - 192;   // 64 threads
            const int items = (p.W - 1) * mb_per_owner;
            const size_t n = size_t(TP_BM) * p.K / 8;   // 16-byte pieces per block
            for (int it = blockIdx.x; it < items; it += gridDim.x) {
                const int d = (p.rank + 1 + it / mb_per_owner) % p.W, blk = it % mb_per_owner;
                uint8_t *dst_base = reinterpret_cast<uint8_t *>(p.peer[d]);
                const size_t row0 = size_t(p.rank) * Mo + size_t(blk) * TP_BM;
                const uint4 *src = reinterpret_cast<const uint4 *>(p.a_shard + size_t(blk) * TP_BM * p.K);
                uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(
                                                            dst_base + (par ? p.off_data[1] : p.off_data[0])) +
                                                        row0 * p.K);
                size_t i = pt;
                for (; i + 3 * 64 < n; i += 4 * 64) {
                    const uint4 v0 = src[i], v1 = src[i + 64], v2 = src[i + 128], v3 = src[i + 192];
                    dst[i] = v0;
                    dst[i + 64] = v1;
                    dst[i + 128] = v2;
                    dst[i + 192] = v3;
                }
                for (; i < n; i += 64) dst[i] = src[i];
                __threadfence_system();
                asm volatile("bar.sync 2, 64;\n" ::: "memory");
                if (pt == 0)
                    st_release_sys(reinterpret_cast<volatile uint32_t *>(dst_base + (par ? p.off_flags[1] : p.off_flags[0])) +
                                       row0 / TP_BM,
                                   epoch);
            }
        }
    } else {
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int local = 0;
        for (int i = blockIdx.x; i < tiles; i += gridDim.x, ++local) {
            int owner, tm, tn, j;
            tile_at(i, owner, tm, tn, j);
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
            const int row = tm * TP_BM + row_in_tile;
            const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
            // RS: a peer's tile goes to its owner's receive slot; an own tile (walked last) meets the peers'
            // partials here: wait for their flags, then sum all W partials in rank order (+ residual) and write the
            // final rows -- no separate reduction pass
            const bool own = MODE == 0 && owner == p.rank;
            const __nv_bfloat16 *recv = reinterpret_cast<const __nv_bfloat16 *>(
                reinterpret_cast<const uint8_t *>(p.peer[p.rank]) + (par ? p.off_data[1] : p.off_data[0]));
            if (own) {
                bool good = true;
                if (lane == 0) {
                    const volatile uint32_t *fl = reinterpret_cast<const volatile uint32_t *>(
                        reinterpret_cast<const uint8_t *>(p.peer[p.rank]) + (par ? p.off_flags[1] : p.off_flags[0]));
                    for (int s = 0; s < p.W && good; ++s)
                        if (s != p.rank) good = tp_wait_flag(fl + size_t(s) * tpo + j, epoch, p.timeout_ns);
                }
                good = __shfl_sync(0xffffffffu, good, 0);
                if (!good) {
                    if (lane == 0) fail();
                    break;
                }
            }
            __nv_bfloat16 *dst_row;
            if (MODE == 0 && !own)
                dst_row = reinterpret_cast<__nv_bfloat16 *>(reinterpret_cast<uint8_t *>(p.peer[owner]) +
                                                           (par ? p.off_data[1] : p.off_data[0])) +
                          (size_t(p.rank) * Mo + (row - owner * Mo)) * p.N;
            else if (own)
                dst_row = p.out + size_t(row - owner * Mo) * p.N;
            else
                dst_row = p.out + size_t(row) * p.N;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32(base + uint32_t(c0), r);
                tc::tmem_ld_wait();
                const int col = tn * BN + c0;
                if (col >= p.N) continue;
                if (own) {   // sum in rank order, this rank's partial from TMEM in its place
                    const int lrow = row - owner * Mo;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        float f[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) f[q] = 0.f;
                        for (int sr = 0; sr < p.W; ++sr) {
                            if (sr == p.rank) {
#pragma unroll
                                for (int q = 0; q < 8; ++q) f[q] += __bfloat162float(__float2bfloat16(__uint_as_float(r[v * 8 + q])));
                            } else if (col + v * 8 + 8 <= p.N) {
                                const uint4 pv = __ldcv(reinterpret_cast<const uint4 *>(
                                    recv + (size_t(sr) * Mo + lrow) * p.N + col + v * 8));
                                const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&pv);
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const float2 g = __bfloat1622float2(p2[q]);
                                    f[2 * q] += g.x;
                                    f[2 * q + 1] += g.y;
                                }
                            }
                        }
                        if (p.residual && col + v * 8 + 8 <= p.N) {
                            const uint4 rv = *reinterpret_cast<const uint4 *>(p.residual + size_t(lrow) * p.N + col + v * 8);
                            const __nv_bfloat162 *r2 = reinterpret_cast<const __nv_bfloat162 *>(&rv);
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float2 g = __bfloat1622float2(r2[q]);
                                f[2 * q] += g.x;
                                f[2 * q + 1] += g.y;
                            }
                        }
                        if (col + v * 8 + 8 <= p.N) {
                            uint4 o;
                            __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                            for (int q = 0; q < 4; ++q) o2[q] = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
                            *reinterpret_cast<uint4 *>(dst_row + col + v * 8) = o;
                        }
                    }
                } else if (col + 32 <= p.N) {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 o;
                        __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            o2[q] = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * q]),
                                                          __uint_as_float(r[v * 8 + 2 * q + 1]));
                        *reinterpret_cast<uint4 *>(dst_row + col + v * 8) = o;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 32; ++q)   // static indices keep r in registers
                        if (col + q < p.N) dst_row[col + q] = __float2bfloat16(__uint_as_float(r[q]));
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[acc]);
            if (MODE == 0 && !own) {   // all four epilogue warps stored the tile: release it to its owner (the
                // barrier orders the warps' peer stores before the flag thread's system fence, which is cumulative)
                asm volatile("bar.sync 1, 128;\n" ::: "memory");
                if (warp == 2 && lane == 0) {
                    __threadfence_system();
                    st_release_sys(reinterpret_cast<volatile uint32_t *>(reinterpret_cast<uint8_t *>(p.peer[owner]) +
                                                                         (par ? p.off_flags[1] : p.off_flags[0])) +
                                       size_t(p.rank) * tpo + j,
                                   epoch);
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * BN);
    }
}

__global__ void tp_bump_epoch(uint32_t *state) { state[0] = state[0] + 1; }

}  // namespace xt

using namespace xt;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tp_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

bool tp_map(CUtensorMap *map, const void *ptr, int rows, int cols, int box_rows) {
    auto fn = tp_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
    cuuint32_t box[2] = {cuuint32_t(TP_BK), cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int MODE>
int tp_launch(const CUtensorMap &ma0, const CUtensorMap &ma1, const CUtensorMap &mb, const CUtensorMap &ml,
              const TpParams &p, cudaStream_t stream) {
    const int smem = TpSmem<BN>::BYTES;
    if (xt_smem_optin(gemm_tp_kernel<BN, MODE>, smem) != cudaSuccess) return -4;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = (p.M / TP_BM) * ((p.N + BN - 1) / BN);
    gemm_tp_kernel<BN, MODE><<<tiles < sms ? tiles : sms, MODE == 1 ? TP_THREADS_AG : TP_THREADS, smem, stream>>>(
        ma0, ma1, mb, ml, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

extern "C" {

// GEMM -> reduce-scatter. a [M, K] and b [N, K] are this rank's K shards (local memory); p.out [M/W, N] receives this
// rank's reduced rows (+ p.residual). Needs M % (128 W) == 0, K % 8 == 0, N % 8 == 0.
int xt_gemm_rs(const void *a, const void *b, const TpParams *pp, cudaStream_t stream) {
    TpParams p = *pp;
    if (p.W < 1 || p.M % (TP_BM * p.W) || p.K % 8 || p.N % 8) return -2;
    CUtensorMap ma, mb;
    const int bn = p.N >= 2048 ? 256 : 128;
    if (!tp_map(&ma, a, p.M, p.K, TP_BM) || !tp_map(&mb, b, p.N, p.K, bn)) return -3;
    int rc = bn == 256 ? tp_launch<256, 0>(ma, ma, mb, ma, p, stream) : tp_launch<128, 0>(ma, ma, mb, ma, p, stream);
    if (rc) return rc;
    tp_bump_epoch<<<1, 1, 0, stream>>>(p.state);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// All-gather -> GEMM. p.a_shard [M/W, K] is this rank's row shard, b [N, K] (this rank's column shard of the layer),
// p.out [M, N]. local_base is this rank's symmetric buffer (host-side value of its address): the GEMM's A tensor maps
// describe its two gather regions, so TMA reads only this rank's memory. Needs M % (128 W) == 0, K % 8, N % 8 == 0.
int xt_ag_gemm(const void *b, const void *local_base, const TpParams *pp, cudaStream_t stream) {
    TpParams p = *pp;
    if (p.W < 1 || p.M % (TP_BM * p.W) || p.K % 8 || p.N % 8 || !local_base) return -2;
    const int Mo = p.M / p.W;
    CUtensorMap ma0, ma1, mb, ml;
    const int bn = p.N >= 2048 ? 256 : 128;
    const uint8_t *base = static_cast<const uint8_t *>(local_base);
    if (!tp_map(&ma0, base + p.off_data[0], p.M, p.K, TP_BM) || !tp_map(&ma1, base + p.off_data[1], p.M, p.K, TP_BM) ||
        !tp_map(&mb, b, p.N, p.K, bn) || !tp_map(&ml, p.a_shard, Mo, p.K, TP_BM))
        return -3;
    int rc = bn == 256 ? tp_launch<256, 1>(ma0, ma1, mb, ml, p, stream) : tp_launch<128, 1>(ma0, ma1, mb, ml, p, stream);
    if (rc) return rc;
    tp_bump_epoch<<<1, 1, 0, stream>>>(p.state);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
