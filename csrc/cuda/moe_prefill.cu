// Grouped FP4 expert GEMM for prefill on the 5th-generation tensor cores (sm_100a: tcgen05 + TMEM + TMA).
//
// Routes are sorted by expert slot (host side), so each slot's tokens form a contiguous run of rows of the gathered
// activations X [R, K] (BF16; each run padded to a multiple of 128 rows). A tile is (run, 128 rows, BN = 128 output
// rows of the expert); the tile list comes from the host. Persistent CTAs, one per SM, 14 warps:
//   warp 0    TMA producer: per k-block of 64, the X tile [128 x 64] BF16 (128-byte swizzle) and the expert's raw
//             FP4 codes [128 rows x 32 bytes] (two boxes of 64 rows: gate and up rows for GATE_UP, consecutive rows
//             for DOWN)
//   warps 6-13 dequantization: E2M1 codes x block scale (E4M3 per 16 or UE8M0 per 32) -> BF16, written in the
//             128-byte-swizzled K-major layout the MMA reads. E2M1 x E4M3 has at most 4 significant bits, so the
//             BF16 weights are exact: the GEMM is W4A16 with FP32 accumulation, the numerics of the decode kernels.
//   warp 1    MMA issuer (kind::f16, M 128, N 128, K 16 per instruction), double-buffered TMEM accumulators
//   warps 2-5 epilogue: GATE_UP -> SwiGLU(g13[0] * gate, g13[1] * up) of the tile's 64 columns -> mid BF16;
//             DOWN -> route weight * g2 * D -> Y FP32 rows (summed per token afterwards in route order)
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA winds down.
// Reference parity: xtier/backend/prefill.py:64-140 (grouped gate/up and down over sorted route tiles with SwiGLU)
// and :1511 (FlashInfer CUTLASS fused MoE on SM100), replaced here by one kernel of this project's own.
#include <cudaTypedefs.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int GP_BM = 128, GP_BN = 128, GP_BK = 64, GP_STAGES = 4, GP_THREADS = 448;
constexpr int GP_DQ_WARPS = 8;   // dequantization warps (6..13)

constexpr int GP_MT = 2;   // m-tiles of 128 rows per work item: every dequantized weight tile feeds GP_MT MMAs

struct GpSmem {
    static constexpr int A1 = GP_BM * GP_BK * 2;         // 16 KB: one m-tile of activations
    static constexpr int A = GP_MT * A1;                  // 32 KB
    static constexpr int RAW = GP_BN * GP_BK / 2;         // 4 KB of codes
    static constexpr int B = GP_BN * GP_BK * 2;           // 16 KB of BF16 weights
    static constexpr int STAGE = A + B + RAW;             // A tiles and B 1024-aligned, RAW after them
    static constexpr int BYTES = GP_STAGES * STAGE + 1024 + 1024;
};

struct GpParams {
    const int32_t *tiles;     // [T, 4]: slot, first row in X, n-tile, valid rows
    int T;
    int K, N_rows;            // K of this GEMM; rows of one expert's weight matrix (2I or H)
    int I;                    // GATE_UP: the expert's intermediate size (up rows start at I)
    int fmt;                  // 0 NVFP4, 1 MXFP4
    const uint8_t *scales;    // [slots, N_rows, K / bs]
    const float *gscale;      // GATE_UP: g13 [slots, 2]; DOWN: g2 [slots]
    const float *route_w;     // DOWN: [R] route weight of each row of X
    const int32_t *dst_row;   // DOWN, optional: [R] the Y row of each row of X (-1: none); null: the same row
    __nv_bfloat16 *mid;       // GATE_UP out: [R, I]
    float *y;                 // DOWN out: [R, H]
    int out_cols;             // I (gate/up) or H (down)
    int *error;
};

template <bool GATE_UP>
__global__ void __launch_bounds__(GP_THREADS, 1)
    moe_grouped_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                       GpParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + GP_STAGES * GpSmem::STAGE);
    uint64_t *ready = full + GP_STAGES;
    uint64_t *empty = ready + GP_STAGES;
    uint64_t *tfull = empty + GP_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = p.K / GP_BK;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < GP_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&ready[s], GP_DQ_WARPS);
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
        tc::tmem_alloc(tmem_slot, 2 * GP_MT * GP_BN);   // two accumulator sets (double buffer) of GP_MT m-tiles
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(p.error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int t = blockIdx.x; t < p.T && !abort_flag; t += gridDim.x) {
                const int4 tl = reinterpret_cast<const int4 *>(p.tiles)[t];
                const int slot = tl.x, row0 = tl.y, nt = tl.z;
                const bool second = tl.w > GP_BM;   // the work item's second m-tile has rows
                const int wrow0 = GATE_UP ? slot * p.N_rows + nt * (GP_BN / 2) : slot * p.N_rows + nt * GP_BN;
                const int wrow1 = GATE_UP ? slot * p.N_rows + p.I + nt * (GP_BN / 2) : wrow0 + GP_BN / 2;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *st = smem + stage * GpSmem::STAGE;
                    uint8_t *raw = st + GpSmem::A + GpSmem::B;
                    tc::mbar_arrive_expect_tx(&full[stage], (second ? 2 : 1) * GpSmem::A1 + GpSmem::RAW);
                    tc::tma_load_2d(st, &tma_x, &full[stage], kb * GP_BK, row0);
                    if (second) tc::tma_load_2d(st + GpSmem::A1, &tma_x, &full[stage], kb * GP_BK, row0 + GP_BM);
                    tc::tma_load_2d(raw, &tma_w, &full[stage], kb * (GP_BK / 2), wrow0);
                    tc::tma_load_2d(raw + GpSmem::RAW / 2, &tma_w, &full[stage], kb * (GP_BK / 2), wrow1);
                    issued = min(issued + 1, GP_STAGES);
                    if (++stage == GP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (abort_flag)
                for (int q = 0; q < issued; ++q) {
                    if (--stage < 0) {
                        stage = GP_STAGES - 1;
                        phase ^= 1;
                    }
                    tc::mbar_wait(&full[stage], phase, 1u << 20);
                }
        }
    } else if (warp >= 6) {
        // dequantization warps: 256 threads, 4 chunks of 8 codes each per k-block (BN rows x 8 chunks); the block
        // scales of a k-block are loaded before waiting for its codes, so their latency hides behind the wait
        const int dt = threadIdx.x - 6 * 32;
        const int bs = p.fmt == 0 ? 16 : 32;
        const int srow = p.K / bs;
        int stage = 0;
        uint32_t phase = 0;
        for (int t = blockIdx.x; t < p.T && !abort_flag; t += gridDim.x) {
            const int4 tl = reinterpret_cast<const int4 *>(p.tiles)[t];
            const int slot = tl.x, nt = tl.z;
            const uint8_t *sp[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = dt + i * 256, r = c >> 3;
                const int wr = GATE_UP ? (r < 64 ? nt * 64 + r : p.I + nt * 64 + (r - 64)) : nt * GP_BN + r;
                sp[i] = p.scales + (size_t(slot) * p.N_rows + wr) * srow;
            }
            // block scales one k-block ahead: the next k-block's loads are in flight while this one is converted
            auto load_sf = [&](int kb, float (&out)[4]) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int kel = kb * GP_BK + ((dt + i * 256) & 7) * 8;
                    out[i] = p.fmt == 0 ? e4m3_to_f(sp[i][kel / 16]) : ue8m0_to_f(sp[i][kel / 32]);
                }
            };
            float sf[4], sfn[4];
            load_sf(0, sf);
            for (int kb = 0; kb < kblocks; ++kb) {
                if (kb + 1 < kblocks) load_sf(kb + 1, sfn);
                bool ok = true;
                if (lane == 0) ok = tc::mbar_wait(&full[stage], phase);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok || abort_flag) {
                    if (lane == 0 && !ok) fail();
                    break;
                }
                uint8_t *st = smem + stage * GpSmem::STAGE;
                uint8_t *bt = st + GpSmem::A;
                const uint8_t *raw = bt + GpSmem::B;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int c = dt + i * 256;   // chunk index: row r, 8-element chunk q
                    const int r = c >> 3, q = c & 7;
                    const uint32_t codes = *reinterpret_cast<const uint32_t *>(raw + r * 32 + q * 4);
                    __half2 h[4];
                    e2m1x8_to_h2(codes, h);
                    uint4 o;
                    __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(h[j]);
                        o2[j] = __floats2bfloat162_rn(f.x * sf[i], f.y * sf[i]);
                    }
                    *reinterpret_cast<uint4 *>(bt + r * 128 + ((q ^ (r & 7)) << 4)) = o;
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&ready[stage]);
                if (++stage == GP_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) sf[i] = sfn[i];
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16_f32(GP_BM, GP_BN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int t = blockIdx.x; t < p.T && !abort_flag; t += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t use = uint32_t(local >> 1);
                if (!tc::mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * GP_MT * GP_BN);
                const bool second = reinterpret_cast<const int4 *>(p.tiles)[t].w > GP_BM;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase) || !tc::mbar_wait(&ready[stage], phase)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * GpSmem::STAGE);
                    const uint64_t ad = tc::sw128_kmajor_desc(sa), bd = tc::sw128_kmajor_desc(sa + GpSmem::A);
                    const uint64_t ad1 = tc::sw128_kmajor_desc(sa + GpSmem::A1);
#pragma unroll
                    for (int k = 0; k < GP_BK / 16; ++k) {
                        tc::mma_f16(d, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        if (second)
                            tc::mma_f16(d + GP_BN, ad1 + uint64_t(2 * k), bd + uint64_t(2 * k), idesc,
                                        (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    tc::mma_commit(&empty[stage]);
                    if (++stage == GP_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit(&tfull[acc]);
            }
        }
    } else {
        // epilogue warps 2-5: TMEM lanes 32*(w%4).. = tile rows
        const int quarter = warp & 3;
        const int rit = quarter * 32 + lane;
        int local = 0;
        for (int t = blockIdx.x; t < p.T; t += gridDim.x, ++local) {
            const int4 tl = reinterpret_cast<const int4 *>(p.tiles)[t];
            const int slot = tl.x, row0 = tl.y, nt = tl.z, valid = tl.w;
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
            for (int mt = 0; mt < GP_MT; ++mt) {
                if (mt > 0 && valid <= mt * GP_BM) break;
                const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * GP_MT * GP_BN + mt * GP_BN);
                const int row = row0 + mt * GP_BM + rit;
                const int vrows = valid - mt * GP_BM;   // rows of this m-tile that hold routes
                if (GATE_UP) {
                    const float gg = p.gscale[2 * slot], gu = p.gscale[2 * slot + 1];
#pragma unroll 1
                    for (int c0 = 0; c0 < 64; c0 += 32) {
                        uint32_t g[32], u[32];
                        tc::tmem_ld32(base + uint32_t(c0), g);
                        tc::tmem_ld32(base + uint32_t(64 + c0), u);
                        tc::tmem_ld_wait();
                        if (rit < vrows) {
                            __nv_bfloat16 *dst = p.mid + size_t(row) * p.out_cols + nt * 64 + c0;
#pragma unroll
                            for (int v = 0; v < 4; ++v) {
                                uint4 o;
                                __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    float h[2];
#pragma unroll
                                    for (int e = 0; e < 2; ++e) {
                                        const float a = __uint_as_float(g[v * 8 + 2 * i + e]) * gg;
                                        const float b = __uint_as_float(u[v * 8 + 2 * i + e]) * gu;
                                        h[e] = a / (1.f + __expf(-a)) * b;
                                    }
                                    o2[i] = __floats2bfloat162_rn(h[0], h[1]);
                                }
                                reinterpret_cast<uint4 *>(dst)[v] = o;
                            }
                        }
                    }
                } else {
                    const float scale = rit < vrows ? p.route_w[row] * p.gscale[slot] : 0.f;
                    const int yrow = rit < vrows ? (p.dst_row ? p.dst_row[row] : row) : -1;
#pragma unroll 1
                    for (int c0 = 0; c0 < GP_BN; c0 += 32) {
                        uint32_t r[32];
                        tc::tmem_ld32(base + uint32_t(c0), r);
                        tc::tmem_ld_wait();
                        if (yrow >= 0) {
                            float *dst = p.y + size_t(yrow) * p.out_cols + nt * GP_BN + c0;
#pragma unroll
                            for (int v = 0; v < 8; ++v)
                                reinterpret_cast<float4 *>(dst)[v] =
                                    make_float4(__uint_as_float(r[4 * v]) * scale, __uint_as_float(r[4 * v + 1]) * scale,
                                                __uint_as_float(r[4 * v + 2]) * scale, __uint_as_float(r[4 * v + 3]) * scale);
                        }
                    }
                }
            }   // m-tiles
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[acc]);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * GP_MT * GP_BN);
    }
}

}  // namespace xt

using namespace xt;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 gp_encode_fn() {
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

}  // namespace

extern "C" {

// One grouped GEMM over the tile list. x [R, K] BF16 (sorted, runs padded to 128 rows), codes [slots * N_rows, K/2],
// scales [slots * N_rows, K/bs]. gate_up: mid [R, I] = SwiGLU(...); else y [R, H] = w * g2 * (x . W2^T).
int xt_moe_grouped(const void *x, int R, const void *codes, int slots, const int32_t *tiles, int T, int gate_up,
                   int K, int N_rows, int I, int fmt, const void *scales, const float *gscale, const float *route_w,
                   const int32_t *dst_row, void *mid, float *y, int out_cols, int *error, cudaStream_t stream) {
    if (T <= 0) return 0;
    if (K % GP_BK || R % GP_BM || N_rows % (gate_up ? 2 : GP_BN) || (gate_up && I % 64)) return -2;
    auto fn = gp_encode_fn();
    if (!fn) return -3;
    CUtensorMap mx, mw;
    {
        cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(R)};
        cuuint64_t strides[1] = {cuuint64_t(K) * 2};
        cuuint32_t box[2] = {GP_BK, GP_BM};
        cuuint32_t estr[2] = {1, 1};
        if (fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -3;
    }
    {
        cuuint64_t dims[2] = {cuuint64_t(K / 2), cuuint64_t(slots) * cuuint64_t(N_rows)};
        cuuint64_t strides[1] = {cuuint64_t(K / 2)};
        cuuint32_t box[2] = {GP_BK / 2, GP_BN / 2};
        cuuint32_t estr[2] = {1, 1};
        if (fn(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(codes), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -3;
    }
    GpParams p{};
    p.tiles = tiles;
    p.T = T;
    p.K = K;
    p.N_rows = N_rows;
    p.I = I;
    p.fmt = fmt;
    p.scales = static_cast<const uint8_t *>(scales);
    p.gscale = gscale;
    p.route_w = route_w;
    p.dst_row = dst_row;
    p.mid = static_cast<__nv_bfloat16 *>(mid);
    p.y = y;
    p.out_cols = out_cols;
    p.error = error;
    {
        const void *f = gate_up ? reinterpret_cast<const void *>(moe_grouped_kernel<true>)
                                : reinterpret_cast<const void *>(moe_grouped_kernel<false>);
        if (xt_smem_optin(f, int(GpSmem::BYTES)) != cudaSuccess) return -4;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = T < sms ? T : sms;
    if (gate_up)
        moe_grouped_kernel<true><<<grid, GP_THREADS, GpSmem::BYTES, stream>>>(mx, mw, p);
    else
        moe_grouped_kernel<false><<<grid, GP_THREADS, GpSmem::BYTES, stream>>>(mx, mw, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ gather / combine
// Around the grouped GEMMs of a prefill call:
// * gather_rows: X[r] = x[src[r]] (BF16 rows; src -1 -> a zero row, the padding of each expert's run), 16-byte copies.
// * route_combine: out[t] = sum over the token's routes j in route order of the route's weighted down row (from the
//   GPU-slot pass Ya or the uploaded-experts pass Yb, whichever computed that route; neither: nothing) + add[t], in
//   FP32, written once as BF16 or FP32. One pass over the route rows instead of a gather, a select and k adds.
namespace xt {

__global__ void __launch_bounds__(256) gather_rows_kernel(const uint4 *__restrict__ x, const int32_t *__restrict__ src,
                                                         uint4 *__restrict__ X, int R, int hv) {
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    if (i >= (long long)R * hv) return;
    const int r = int(i / hv), c = int(i % hv);
    const int s = src[r];
    X[i] = s >= 0 ? x[size_t(s) * hv + c] : make_uint4(0, 0, 0, 0);
}

template <bool OUT_F32>
__global__ void __launch_bounds__(256) route_combine_kernel(const float *__restrict__ Ya, const int32_t *__restrict__ da,
                                                           int ka, const float *__restrict__ Yb,
                                                           const int32_t *__restrict__ db, int kb,
                                                           const __nv_bfloat16 *__restrict__ add, void *out, int m,
                                                           int H) {
    const int hv = H / 4;
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    if (i >= (long long)m * hv) return;
    const int t = int(i / hv), c = int(i % hv);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const int kk = ka > kb ? ka : kb;
    for (int j = 0; j < kk; ++j) {
        const int ra = j < ka ? da[size_t(t) * ka + j] : -1;
        const int rb = (ra < 0 && Yb && j < kb) ? db[size_t(t) * kb + j] : -1;
        const float *row = ra >= 0 ? Ya + size_t(ra) * H : (rb >= 0 ? Yb + size_t(rb) * H : nullptr);
        if (row) {
            const float4 v = reinterpret_cast<const float4 *>(row)[c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
    }
    if (add) {
        const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(add + size_t(t) * H + 4 * c);
        const float2 p = __bfloat1622float2(a2[0]), q = __bfloat1622float2(a2[1]);
        acc.x += p.x;
        acc.y += p.y;
        acc.z += q.x;
        acc.w += q.y;
    }
    if (OUT_F32) {
        reinterpret_cast<float4 *>(out)[i] = acc;
    } else {
        __nv_bfloat162 o[2] = {__floats2bfloat162_rn(acc.x, acc.y), __floats2bfloat162_rn(acc.z, acc.w)};
        reinterpret_cast<uint2 *>(out)[i] = *reinterpret_cast<uint2 *>(o);
    }
}

}  // namespace xt

extern "C" int xt_gather_rows(const void *x, const int32_t *src, void *X, int R, int H, cudaStream_t stream) {
    if (H % 8 || R < 0) return -2;
    if (R == 0) return 0;
    const int hv = H / 8;
    const long long th = (long long)R * hv;
    xt::gather_rows_kernel<<<unsigned((th + 255) / 256), 256, 0, stream>>>(static_cast<const uint4 *>(x), src,
                                                                           static_cast<uint4 *>(X), R, hv);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int xt_route_combine(const float *Ya, const int32_t *da, int ka, const float *Yb, const int32_t *db, int kb,
                                const void *add, void *out, int out_f32, int m, int H, cudaStream_t stream) {
    if (H % 4 || m < 0 || ka < 1 || (Yb && kb < 1)) return -2;
    if (m == 0) return 0;
    const long long th = (long long)m * (H / 4);
    const unsigned grid = unsigned((th + 255) / 256);
    auto A = static_cast<const __nv_bfloat16 *>(add);
    if (out_f32)
        xt::route_combine_kernel<true><<<grid, 256, 0, stream>>>(Ya, da, ka, Yb, db, kb, A, out, m, H);
    else
        xt::route_combine_kernel<false><<<grid, 256, 0, stream>>>(Ya, da, ka, Yb, db, kb, A, out, m, H);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
