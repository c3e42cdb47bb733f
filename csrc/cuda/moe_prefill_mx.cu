// Block-scaled grouped expert GEMM for prefill: MXFP4 expert weights x MXFP8 activations on tcgen05
// (kind::mxf8f6f4.block_scale, E4M3 x E2M1 with UE8M0 scales per 32 values along K, FP32 accumulation in TMEM): the
// numerics of the reference's FP4 prefill (MXFP4 weights, MXFP8 activations), at the FP8 tensor rate instead of the
// BF16 rate of the W4A16 kernel in moe_prefill.cu, which stays as the exact option.
//
// Same work list as moe_grouped (routes sorted by slot, runs padded to 128 rows), one 128-row m-tile per item.
// The activations come pre-quantized (mx_quant_rows: E4M3 rows X8 [R, K] and their scales SFX laid out per
// (m-tile, 128-column k-block) as the 512-byte scale atom the MMA reads, see below). Persistent CTAs, 10 warps:
//   warp 0     TMA producer, six stages deep: per k-block of 128, the X8 tile [128 x 128 bytes] (128-byte swizzle),
//              its 512 scale bytes (one bulk copy) and the expert's E2M1 codes for 128 weight rows (gate and up rows
//              for GATE_UP, consecutive rows for DOWN) through a tensor map of type 16U4_ALIGN16B: TMA places every
//              8 bytes of packed codes in a 16-byte slot (the operand layout the MMA reads for E2M1 under
//              kind::mxf8f6f4), swizzled like the activations, so the weights need no conversion pass
//   warps 6-9  scale warps, one weight row per thread: the row's UE8M0 scale word of the k-block (read from global
//              memory four to eight k-blocks ahead) into the weight scale atom
//   warp 1     TMEM owner (512 columns) and MMA issuer: per k-block both scale atoms go to TMEM (tcgen05.cp
//              32x128b.warpx4), then four MMAs of 128 x 128 x 32, each selecting its byte of the scale words; two
//              accumulator buffers so the epilogue of one item overlaps the next
//   warps 2-5  epilogue, as moe_grouped: GATE_UP -> SwiGLU(g13[0] * gate, g13[1] * up) -> mid BF16; DOWN -> route
//              weight * g2 * D -> Y FP32 rows
// Scale atom (128 rows x 4 scales of one k-block, 512 bytes): byte (r % 32) * 16 + (r / 32) * 4 + j holds row r's
// scale of K values [32 j, 32 j + 32). tcgen05.cp 32x128b.warpx4 copies its 32 rows of 16 bytes to 4 TMEM columns of
// every lane quarter; the MMA reads row r's scale word in lane r, column r / 32, and the byte named by the two top bits
// of the scale address (the idesc's scale-factor id).
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA winds down.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "mx_common.cuh"
#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int MX_BM = 128, MX_BN = 128, MX_BK = 128, MX_STAGES = 6, MX_THREADS = 320;
constexpr int MX_SC_WARPS = 4;              // scale warps (6..9)
constexpr uint32_t MX_SF_COL = 256;         // TMEM column of the scale atoms: 8 columns per stage (X then W)

struct MxSmem {
    static constexpr int A = MX_BM * MX_BK;       // 16 KB of E4M3 activations
    static constexpr int B = MX_BN * MX_BK;       // 16 KB: E2M1 weights, 16 codes per 16-byte slot
    static constexpr int B_TX = B / 2;            // bytes the TMA counts for them (the packed codes)
    static constexpr int SF = 512;                // one scale atom
    static constexpr int STAGE = A + B + 2 * SF;  // A, B 1024-aligned; the two atoms after them
    static constexpr int BYTES = MX_STAGES * STAGE + 1024 + 1024;
};

struct MxParams {
    const int32_t *tiles;     // [T, 4]: slot, first row in X, n-tile, valid rows (<= 128)
    int T;
    int K, N_rows, I;
    const uint8_t *sfx;       // [R / 128][K / 128][512] activation scale atoms
    const uint8_t *codes;     // [slots, N_rows, K / 2] E2M1
    const uint8_t *scales;    // [slots, N_rows, K / 32] UE8M0
    const float *gscale;      // GATE_UP: g13 [slots, 2]; DOWN: g2 [slots]
    const float *route_w;     // DOWN: [R]
    const int32_t *dst_row;   // DOWN, optional: [R] the Y row of each row of X (-1: none)
    __nv_bfloat16 *mid;       // GATE_UP out: [R, I]
    float *y;                 // DOWN out: [rows, H]
    int out_cols;
    int *error;
};

template <bool GATE_UP>
__global__ void __launch_bounds__(MX_THREADS, 1)
    moe_grouped_mx_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                          MxParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + MX_STAGES * MxSmem::STAGE);
    uint64_t *ready = full + MX_STAGES;
    uint64_t *empty = ready + MX_STAGES;
    uint64_t *tfull = empty + MX_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = p.K / MX_BK;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < MX_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&ready[s], MX_SC_WARPS);
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
                const uint8_t *sfx = p.sfx + size_t(row0 / MX_BM) * kblocks * MxSmem::SF;
                const int wrow0 = GATE_UP ? slot * p.N_rows + nt * (MX_BN / 2) : slot * p.N_rows + nt * MX_BN;
                const int wrow1 = GATE_UP ? slot * p.N_rows + p.I + nt * (MX_BN / 2) : wrow0 + MX_BN / 2;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *st = smem + stage * MxSmem::STAGE;
                    tc::mbar_arrive_expect_tx(&full[stage], MxSmem::A + MxSmem::B_TX + MxSmem::SF);
                    tc::tma_load_2d(st, &tma_x, &full[stage], kb * MX_BK, row0);
                    tc::tma_load_2d(st + MxSmem::A, &tma_w, &full[stage], kb * MX_BK, wrow0);
                    tc::tma_load_2d(st + MxSmem::A + MxSmem::B / 2, &tma_w, &full[stage], kb * MX_BK, wrow1);
                    mx_bulk_g2s(st + MxSmem::A + MxSmem::B, sfx + size_t(kb) * MxSmem::SF, MxSmem::SF, &full[stage]);
                    issued = min(issued + 1, MX_STAGES);
                    if (++stage == MX_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (abort_flag)   // let the copies in flight land before the CTA exits
                for (int q = 0; q < issued; ++q) {
                    if (--stage < 0) {
                        stage = MX_STAGES - 1;
                        phase ^= 1;
                    }
                    tc::mbar_wait(&full[stage], phase, 1u << 20);
                }
        }
    } else if (warp >= 6) {
        // scale warps: thread r owns weight-tile row r; scale words of a group of four k-blocks in registers, the
        // next group's in flight (copied into place four k-blocks after their loads were issued)
        const int r = threadIdx.x - 6 * 32;
        const size_t srow = size_t(p.K) / 32;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.T && ok && !abort_flag; t += gridDim.x) {
            const int4 tl = reinterpret_cast<const int4 *>(p.tiles)[t];
            const int slot = tl.x, nt = tl.z;
            const int wr = GATE_UP ? (r < 64 ? nt * 64 + r : p.I + nt * 64 + (r - 64)) : nt * MX_BN + r;
            // one word per k-block: rows are 4-byte aligned since K % 128 == 0
            const uint32_t *sp = reinterpret_cast<const uint32_t *>(p.scales + (size_t(slot) * p.N_rows + wr) * srow);
            uint32_t cur[4], nxt[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                cur[j] = j < kblocks ? sp[j] : 0u;
                nxt[j] = 4 + j < kblocks ? sp[4 + j] : 0u;
            }
            for (int g = 0; g < kblocks && ok; g += 4) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (g + j >= kblocks) break;
                    int good = 1;
                    if (lane == 0) good = tc::mbar_wait(&full[stage], phase);
                    good = __shfl_sync(0xffffffffu, good, 0);
                    if (!good || abort_flag) {
                        if (lane == 0 && !good) fail();
                        ok = false;
                        break;
                    }
                    *reinterpret_cast<uint32_t *>(smem + stage * MxSmem::STAGE + MxSmem::A + MxSmem::B + MxSmem::SF +
                                                  (r & 31) * 16 + (r >> 5) * 4) = cur[j];
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&ready[stage]);
                    if (++stage == MX_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    cur[j] = nxt[j];
                    nxt[j] = g + 8 + j < kblocks ? sp[g + 8 + j] : 0u;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
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
                const uint32_t d = tmem + uint32_t(acc * MX_BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!tc::mbar_wait(&full[stage], phase) || !tc::mbar_wait(&ready[stage], phase)) {
                        fail();
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * MxSmem::STAGE);
                    const uint32_t sfa = tmem + MX_SF_COL + uint32_t(stage * 8), sfb = sfa + 4;
                    sf_copy(sfa, sf_atom_desc(sa + MxSmem::A + MxSmem::B));
                    sf_copy(sfb, sf_atom_desc(sa + MxSmem::A + MxSmem::B + MxSmem::SF));
                    const uint64_t ad = tc::sw128_kmajor_desc(sa), bd = tc::sw128_kmajor_desc(sa + MxSmem::A);
#pragma unroll
                    for (int k = 0; k < MX_BK / 32; ++k)   // K = 32 bytes per MMA; byte k of the scale words
                        mma_mx(d, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc_mx(MX_BM, MX_BN, uint32_t(k), MX_FMT_E2M1),
                               sfa | (uint32_t(k) << 30), sfb | (uint32_t(k) << 30), (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&empty[stage]);
                    if (++stage == MX_STAGES) {
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
            const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * MX_BN);
            const int row = row0 + rit;
            if (GATE_UP) {
                const float gg = p.gscale[2 * slot], gu = p.gscale[2 * slot + 1];
#pragma unroll 1
                for (int c0 = 0; c0 < 64; c0 += 32) {
                    uint32_t g[32], u[32];
                    tc::tmem_ld32(base + uint32_t(c0), g);
                    tc::tmem_ld32(base + uint32_t(64 + c0), u);
                    tc::tmem_ld_wait();
                    if (rit < valid) {
                        __nv_bfloat16 *dst = p.mid + size_t(row) * p.out_cols + nt * 64 + c0;
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 o;
                            __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                float hh[2];
#pragma unroll
                                for (int e = 0; e < 2; ++e) {
                                    const float a = __uint_as_float(g[v * 8 + 2 * i + e]) * gg;
                                    const float b = __uint_as_float(u[v * 8 + 2 * i + e]) * gu;
                                    hh[e] = a / (1.f + __expf(-a)) * b;
                                }
                                o2[i] = __floats2bfloat162_rn(hh[0], hh[1]);
                            }
                            reinterpret_cast<uint4 *>(dst)[v] = o;
                        }
                    }
                }
            } else {
                const float scale = rit < valid ? p.route_w[row] * p.gscale[slot] : 0.f;
                const int yrow = rit < valid ? (p.dst_row ? p.dst_row[row] : row) : -1;
#pragma unroll 1
                for (int c0 = 0; c0 < MX_BN; c0 += 32) {
                    uint32_t r[32];
                    tc::tmem_ld32(base + uint32_t(c0), r);
                    tc::tmem_ld_wait();
                    if (yrow >= 0) {
                        float *dst = p.y + size_t(yrow) * p.out_cols + nt * MX_BN + c0;
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            reinterpret_cast<float4 *>(dst)[v] =
                                make_float4(__uint_as_float(r[4 * v]) * scale, __uint_as_float(r[4 * v + 1]) * scale,
                                            __uint_as_float(r[4 * v + 2]) * scale, __uint_as_float(r[4 * v + 3]) * scale);
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

// Rows of X (BF16 [*, K], row src[r] of x, or zeros for src[r] < 0) -> MXFP8: E4M3 x8 [R, K] and the scale atoms
// sfx [R / 128][K / 128][512]. One thread per 32 values: s = 2^ceil(log2(amax / 448)) (no value saturates), UE8M0
// byte log2(s) + 127, x8 = E4M3(x / s) rounded to nearest even.
__global__ void __launch_bounds__(256) mx_quant_rows_kernel(const __nv_bfloat16 *__restrict__ x,
                                                           const int32_t *__restrict__ src, int R, int K,
                                                           uint8_t *__restrict__ x8, uint8_t *__restrict__ sfx) {
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    const int nb = K / 32;
    if (i >= (long long)R * nb) return;
    const int r = int(i / nb), b = int(i % nb);
    const int s = src ? src[r] : r;
    float v[32];
    if (s >= 0) {
        const uint4 *p = reinterpret_cast<const uint4 *>(x + size_t(s) * K + b * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 w = p[q];
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&ws[e]));
                v[q * 8 + 2 * e] = f.x;
                v[q * 8 + 2 * e + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
    int E = -127;
    if (amax > 0.f) {
        const uint32_t bits = __float_as_uint(amax / 448.f);
        E = int((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) ? 1 : 0);
        E = max(-126, min(127, E));
        if (amax * __uint_as_float(uint32_t(127 - E) << 23) > 448.f && E < 127) ++E;
    }
    const float inv = E > -127 ? __uint_as_float(uint32_t(127 - E) << 23) : 0.f;   // 2^-E (E >= -126)
    uint32_t out[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
            uint16_t pr;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n"
                : "=h"(pr)
                : "f"(v[w * 4 + e + 1] * inv), "f"(v[w * 4 + e] * inv));
            word |= uint32_t(pr) << (8 * e);
        }
        out[w] = word;
    }
    uint4 *dst = reinterpret_cast<uint4 *>(x8 + size_t(r) * K + b * 32);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    const int kb = b >> 2, j = b & 3, rr = r & 127;
    sfx[(size_t(r >> 7) * (K / MX_BK) + kb) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + j] = uint8_t(E + 127);
}

}  // namespace xt

using namespace xt;

extern "C" {

int xt_mx_quant_rows(const void *x, const int32_t *src, int R, int K, void *x8, void *sfx, cudaStream_t stream) {
    if (R <= 0) return 0;
    if (K % MX_BK || R % MX_BM) return -2;
    const long long n = (long long)R * (K / 32);
    mx_quant_rows_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(x), src, R,
                                                                        K, static_cast<uint8_t *>(x8),
                                                                        static_cast<uint8_t *>(sfx));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// tiles [T, 4] as moe_grouped, with items of at most 128 rows. x8 [R, K] E4M3 + sfx atoms (xt_mx_quant_rows);
// codes / scales the MXFP4 slot pool; GATE_UP writes mid [R, I] BF16, DOWN y (rows of dst_row, or R) FP32.
int xt_moe_grouped_mx(const void *x8, const void *sfx, int R, const void *codes, const void *scales, int slots,
                      const int32_t *tiles, int T, int gate_up, int K, int N_rows, int I, const float *gscale,
                      const float *route_w, const int32_t *dst_row, void *mid, float *y, int out_cols, int *error,
                      cudaStream_t stream) {
    if (T <= 0) return 0;
    if (K % MX_BK || R % MX_BM || N_rows % (gate_up ? 2 : MX_BN) || (gate_up && I % 64) || slots <= 0) return -2;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult qr;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return -3;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    CUtensorMap mx;
    {
        cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(R)};
        cuuint64_t strides[1] = {cuuint64_t(K)};
        cuuint32_t box[2] = {MX_BK, MX_BM};
        cuuint32_t estr[2] = {1, 1};
        if (fn(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(x8), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -3;
    }
    CUtensorMap mw;
    {
        // elements: K codes per row (packed, K / 2 bytes); box 128 codes x 64 rows -> 64 rows of 128 bytes in smem
        if (reinterpret_cast<uintptr_t>(codes) % 32 || (K / 2) % 32) return -2;
        cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(slots) * cuuint64_t(N_rows)};
        cuuint64_t strides[1] = {cuuint64_t(K / 2)};
        cuuint32_t box[2] = {MX_BK, MX_BN / 2};
        cuuint32_t estr[2] = {1, 1};
        if (fn(&mw, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void *>(codes), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -3;
    }
    MxParams p{};
    p.tiles = tiles;
    p.T = T;
    p.K = K;
    p.N_rows = N_rows;
    p.I = I;
    p.sfx = static_cast<const uint8_t *>(sfx);
    p.codes = static_cast<const uint8_t *>(codes);
    p.scales = static_cast<const uint8_t *>(scales);
    p.gscale = gscale;
    p.route_w = route_w;
    p.dst_row = dst_row;
    p.mid = static_cast<__nv_bfloat16 *>(mid);
    p.y = y;
    p.out_cols = out_cols;
    p.error = error;
    const void *f = gate_up ? reinterpret_cast<const void *>(moe_grouped_mx_kernel<true>)
                            : reinterpret_cast<const void *>(moe_grouped_mx_kernel<false>);
    if (xt_smem_optin(f, int(MxSmem::BYTES)) != cudaSuccess) return -4;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::min(T, sms);
    if (gate_up)
        moe_grouped_mx_kernel<true><<<grid, MX_THREADS, MxSmem::BYTES, stream>>>(mx, mw, p);
    else
        moe_grouped_mx_kernel<false><<<grid, MX_THREADS, MxSmem::BYTES, stream>>>(mx, mw, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
