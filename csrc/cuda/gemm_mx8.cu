// Dense W8A8 GEMM on the block-scaled tensor cores (MXFP8): y [M, N] BF16 (+ an optional BF16 residual) =
// x8 [M, K] . w8 [N, K]^T with E4M3 operands and UE8M0 scales per 32 values along K (tcgen05 kind::mxf8f6f4, FP32
// accumulation in TMEM). Both operands come quantized in the layout mx_quant_rows writes (row-major E4M3, and the
// 512-byte scale atoms per (128-row tile, 128-wide k-block), see mx_common.cuh): the activations per call, the
// weights once at load, so neither scale needs a register pass. This is the B200 form of the reference's W8A8 prefill
// GEMM (xtier/packs/glm5_next/fp8_weights.py: E4M3 weights and per-token activation groups of 128 with FP32 scales,
// group dots scaled in FP32): the block scales are applied inside the MMA instead of per group in registers.
//
// Persistent CTAs over the (m-tile, n-tile) grid in grouped order (tc::tile_coords), 6 warps:
//   warp 0     TMA producer, MG_STAGES deep: per k-block the x8 and w8 tiles (128 x 128 bytes each, 128-byte
//              swizzle) and both scale atoms (untiled bulk copies)
//   warp 1     TMEM owner (512 columns) and MMA issuer: both atoms into TMEM (tcgen05.cp 32x128b.warpx4), four MMAs of
//              128 x 128 x 32 per k-block, each naming its byte of the scale words; two accumulators, so the epilogue
//              of one tile overlaps the next tile's MMAs
//   warps 2-5  epilogue: one tile row per thread, FP32 accumulator (+ residual) -> BF16 row of y
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA winds down.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "mx_common.cuh"
#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int MG_BM = 128, MG_BN = 128, MG_BK = 128, MG_STAGES = 6, MG_THREADS = 192, MG_GROUP_M = 8;
constexpr uint32_t MG_SF_COL = 256;   // TMEM column of the scale atoms: 8 columns per stage (x then w)

struct MgSmem {
    static constexpr int A = MG_BM * MG_BK;       // 16 KB of E4M3 activations
    static constexpr int B = MG_BN * MG_BK;       // 16 KB of E4M3 weights
    static constexpr int SF = 512;                // one scale atom
    static constexpr int STAGE = A + B + 2 * SF;  // A, B 1024-aligned; the two atoms after them
    static constexpr int BYTES = MG_STAGES * STAGE + 1024 + 1024;
};

__global__ void __launch_bounds__(MG_THREADS, 1)
    gemm_mx8_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                    const uint8_t *__restrict__ sfx, const uint8_t *__restrict__ sfw, int M, int N, int K,
                    const __nv_bfloat16 *__restrict__ residual, __nv_bfloat16 *__restrict__ y, int *error) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + MG_STAGES * MgSmem::STAGE);
    uint64_t *empty = full + MG_STAGES;
    uint64_t *tfull = empty + MG_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = K / MG_BK;
    const int tiles_m = (M + MG_BM - 1) / MG_BM, tiles_n = N / MG_BN, tiles = tiles_m * tiles_n;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < MG_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 4);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_x);
        tc::prefetch_tmap(&tma_w);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    pdl_wait();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x) {
                int tm, tn;
                tc::tile_coords(t, tiles_m, tiles_n, MG_GROUP_M, tm, tn);
                const uint8_t *ax = sfx + size_t(tm) * kblocks * MgSmem::SF;
                const uint8_t *aw = sfw + size_t(tn) * kblocks * MgSmem::SF;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *st = smem + stage * MgSmem::STAGE;
                    tc::mbar_arrive_expect_tx(&full[stage], MgSmem::A + MgSmem::B + 2 * MgSmem::SF);
                    tc::tma_load_2d(st, &tma_x, &full[stage], kb * MG_BK, tm * MG_BM);
                    tc::tma_load_2d(st + MgSmem::A, &tma_w, &full[stage], kb * MG_BK, tn * MG_BN);
                    mx_bulk_g2s(st + MgSmem::A + MgSmem::B, ax + size_t(kb) * MgSmem::SF, MgSmem::SF, &full[stage]);
                    mx_bulk_g2s(st + MgSmem::A + MgSmem::B + MgSmem::SF, aw + size_t(kb) * MgSmem::SF, MgSmem::SF,
                                &full[stage]);
                    issued = min(issued + 1, MG_STAGES);
                    if (++stage == MG_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (abort_flag)   // let the copies in flight land before the CTA exits
                for (int q = 0; q < issued; ++q) {
                    if (--stage < 0) {
                        stage = MG_STAGES - 1;
                        phase ^= 1;
                    }
                    tc::mbar_wait(&full[stage], phase, 1u << 20);
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t use = uint32_t(local >> 1);
                if (!tc::mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * MG_BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * MgSmem::STAGE);
                    const uint32_t sfa = tmem + MG_SF_COL + uint32_t(stage * 8), sfb = sfa + 4;
                    sf_copy(sfa, sf_atom_desc(sa + MgSmem::A + MgSmem::B));
                    sf_copy(sfb, sf_atom_desc(sa + MgSmem::A + MgSmem::B + MgSmem::SF));
                    const uint64_t ad = tc::sw128_kmajor_desc(sa), bd = tc::sw128_kmajor_desc(sa + MgSmem::A);
#pragma unroll
                    for (int k = 0; k < MG_BK / 32; ++k)   // K = 32 bytes per MMA; byte k of the scale words
                        mma_mx(d, ad + uint64_t(2 * k), bd + uint64_t(2 * k),
                               idesc_mx(MG_BM, MG_BN, uint32_t(k), MX_FMT_E4M3), sfa | (uint32_t(k) << 30),
                               sfb | (uint32_t(k) << 30), (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&empty[stage]);
                    if (++stage == MG_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit(&tfull[acc]);
            }
        }
    } else {
        // epilogue warps 2-5: TMEM lanes 32 * (w % 4).. = tile rows
        const int quarter = warp & 3;
        const int rit = quarter * 32 + lane;
        int local = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
            int tm, tn;
            tc::tile_coords(t, tiles_m, tiles_n, MG_GROUP_M, tm, tn);
            const int acc = local & 1;
            const uint32_t use = uint32_t(local >> 1);
            bool ok = true;
            if (lane == 0) ok = tc::mbar_wait(&tfull[acc], use & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_flag) {
                if (lane == 0 && !ok) fail();
                break;
            }
            __syncwarp();
            tc::tc_fence_after();
            const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * MG_BN);
            const int row = tm * MG_BM + rit;
#pragma unroll 1
            for (int c0 = 0; c0 < MG_BN; c0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32(base + uint32_t(c0), r);
                tc::tmem_ld_wait();
                if (row < M) {
                    const size_t off = size_t(row) * N + size_t(tn) * MG_BN + c0;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        float add[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                        if (residual) {
                            const uint4 rw = reinterpret_cast<const uint4 *>(residual + off)[v];
                            const __nv_bfloat162 *r2 = reinterpret_cast<const __nv_bfloat162 *>(&rw);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float2 f = __bfloat1622float2(r2[i]);
                                add[2 * i] = f.x;
                                add[2 * i + 1] = f.y;
                            }
                        }
                        uint4 o;
                        __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            o2[i] = __floats2bfloat162_rn(__uint_as_float(r[8 * v + 2 * i]) + add[2 * i],
                                                          __uint_as_float(r[8 * v + 2 * i + 1]) + add[2 * i + 1]);
                        reinterpret_cast<uint4 *>(y + off)[v] = o;
                    }
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
        tc::tmem_dealloc(tmem, 512);
    }
}

}  // namespace xt

using namespace xt;

extern "C" {

// y [M, N] BF16 (+ residual [M, N] BF16 when given) = x8 [Mp, K] . w8 [N, K]^T, both MXFP8 in the layout of
// xt_mx_quant_rows (sfx [Mp / 128][K / 128][512], sfw [N / 128][K / 128][512]); Mp = M rounded up to 128 (the quantized
// rows past M are read and dropped). K % 128 == 0, N % 128 == 0.
int xt_gemm_mx8(const void *x8, const void *sfx, int M, const void *w8, const void *sfw, int N, int K,
                const void *residual, void *y, int *error, cudaStream_t stream) {
    if (M <= 0) return 0;
    if (K % MG_BK || N % MG_BN || K <= 0 || N <= 0) return -2;
    if (reinterpret_cast<uintptr_t>(x8) % 16 || reinterpret_cast<uintptr_t>(w8) % 16 ||
        reinterpret_cast<uintptr_t>(sfx) % 16 || reinterpret_cast<uintptr_t>(sfw) % 16 ||
        reinterpret_cast<uintptr_t>(y) % 16 || reinterpret_cast<uintptr_t>(residual) % 16)
        return -2;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult qr;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return -3;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    const int Mp = (M + MG_BM - 1) / MG_BM * MG_BM;
    auto map = [&](CUtensorMap *m, const void *p, int rows) {
        cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
        cuuint64_t strides[1] = {cuuint64_t(K)};
        cuuint32_t box[2] = {MG_BK, 128};
        cuuint32_t estr[2] = {1, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(p), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    CUtensorMap mx, mw;
    if (!map(&mx, x8, Mp) || !map(&mw, w8, N)) return -3;
    if (xt_smem_optin(gemm_mx8_kernel, int(MgSmem::BYTES)) != cudaSuccess) return -4;
    int sms = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int tiles = (Mp / MG_BM) * (N / MG_BN);
    const cudaError_t e = xt_launch(gemm_mx8_kernel, dim3(tiles < sms ? tiles : sms), dim3(MG_THREADS),
                                    size_t(MgSmem::BYTES), stream, mx, mw, static_cast<const uint8_t *>(sfx),
                                    static_cast<const uint8_t *>(sfw), M, N, K,
                                    static_cast<const __nv_bfloat16 *>(residual), static_cast<__nv_bfloat16 *>(y),
                                    error);
    return e == cudaSuccess ? 0 : -1;
}

}  // extern "C"
