// DeepSeek-style MLA attention over an NVFP4 latent KV cache, decode path (sm_100a):
//
//   mla_kv_write    one warp per new token: the 512 latent values -> NVFP4 (E2M1 codes + one E4M3 scale per 16,
//                   global scale 1), the 64 rotary values stay BF16. 416 bytes per token instead of 1152.
//   mla_gather      the selected keys of each query (an index list per query: the DSA indexer's top-k, or 0..n-1 for
//                   dense attention) dequantized into a K tile [keys, 576] and a transposed V tile [512, keys], BF16,
//                   the operand layouts of the tensor-core kernel below (both K-major).
//   mla_attend      one CTA per (query, block of 128 selected keys), tcgen05 + TMEM + TMA:
//                     S[128 heads, 128 keys] = Q[128, 576] . K^T            (9 k-blocks of 64, TMEM columns 256..383)
//                     P = exp2(S * scale - rowmax) in BF16, written to shared memory in the 128-byte-swizzled
//                         K-major layout the MMA reads (4 softmax warps, one head row per thread)
//                     O[128, 512] = P . V                                    (two N = 256 halves: TMEM columns 0..255
//                                                                             and 256..511 -- the second reuses S's)
//                   and writes the unnormalized O with the row max and sum; a block is one softmax pass, so no
//                   accumulator rescaling is needed inside the CTA.
//   mla_merge       per (query, head): the blocks' partials -> softmax-weighted sum -> BF16 latent output [128, 512]
//                   (the per-head value projection W_uv follows as a batched GEMM).
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA winds down.
// Reference parity: xtier/packs/deepseek_v4/sparse_mla.py:1-20 (sparse MLA over a quantized KV cache: BF16 tensor-core
// Q.K with FP32 scores, P in BF16 for the PV product, FP32 accumulation, split keys merged in FP32; invalid indices
// (-1) never enter the sums).
#include <cudaTypedefs.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int MLA_H = 128;       // heads (the UMMA M)
constexpr int MLA_L = 512;       // latent dims
constexpr int MLA_R = 64;        // rotary dims
constexpr int MLA_D = MLA_L + MLA_R;
constexpr int MLA_BK = 64;       // k-block (one 128-byte swizzle row of BF16)
constexpr int MLA_NB = 128;      // selected keys per CTA
constexpr int MLA_STAGES = 4;
constexpr int MLA_THREADS = 192; // warp 0 TMA, warp 1 MMA, warps 2-5 softmax / epilogue

// ------------------------------------------------------------------------------------------------ cache write
__global__ void __launch_bounds__(256) mla_kv_write_kernel(const __nv_bfloat16 *__restrict__ lat, const int64_t *slot,
                                                           uint8_t *codes, uint8_t *scales, __nv_bfloat16 *rope,
                                                           int T) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const __nv_bfloat16 *x = lat + size_t(warp) * MLA_D;
    const size_t s = size_t(slot[warp]);
    // lane = one block of 16 latent values
    float v[16];
    const uint4 *src = reinterpret_cast<const uint4 *>(x + lane * 16);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 u = src[c];
        const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(b[i]);
            v[c * 8 + 2 * i] = f.x;
            v[c * 8 + 2 * i + 1] = f.y;
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint8_t sc = f32_to_e4m3(amax / 6.f);
    const float sf = e4m3_to_f(sc);
    const float inv = sf > 0.f ? 1.f / sf : 0.f;
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc |= uint32_t(f32x2_to_e2m1(v[h * 8 + 2 * i] * inv, v[h * 8 + 2 * i + 1] * inv)) << (8 * i);
        w[h] = acc;
    }
    *reinterpret_cast<uint2 *>(codes + s * (MLA_L / 2) + lane * 8) = make_uint2(w[0], w[1]);
    scales[s * (MLA_L / 16) + lane] = sc;
    reinterpret_cast<__nv_bfloat162 *>(rope + s * MLA_R)[lane] =
        reinterpret_cast<const __nv_bfloat162 *>(x + MLA_L)[lane];
}

// ------------------------------------------------------------------------------------------------ gather
// grid (blocks of 32 selected keys, queries); idx [Q, nsel] int32 slots (-1: none). Kg [Q, nsel, 576], Vt [Q, 512,
// nsel]. The block's latent rows are staged in shared memory so the transposed V rows are written 64 bytes at a time.
__global__ void __launch_bounds__(256) mla_gather_kernel(const int32_t *__restrict__ idx, int nsel,
                                                         const uint8_t *__restrict__ codes,
                                                         const uint8_t *__restrict__ scales,
                                                         const __nv_bfloat16 *__restrict__ rope,
                                                         __nv_bfloat16 *__restrict__ Kg, __nv_bfloat16 *__restrict__ Vt) {
    __shared__ __align__(16) __nv_bfloat16 tile[32][MLA_L + 8];
    const int q = blockIdx.y, j0 = blockIdx.x * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int jj = warp; jj < 32; jj += 8) {
        const int j = j0 + jj;
        const int s = j < nsel ? idx[size_t(q) * nsel + j] : -1;
        __nv_bfloat16 *krow = Kg + (size_t(q) * nsel + min(j, nsel - 1)) * MLA_D;
        // lane: 16 latent values (8 code bytes, one scale)
        __nv_bfloat162 out[8];
        if (s >= 0) {
            const uint2 cw = *reinterpret_cast<const uint2 *>(codes + size_t(s) * (MLA_L / 2) + lane * 8);
            const float sf = e4m3_to_f(scales[size_t(s) * (MLA_L / 16) + lane]);
            __half2 h[4];
            e2m1x8_to_h2(cw.x, h);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h[i]);
                out[i] = __floats2bfloat162_rn(f.x * sf, f.y * sf);
            }
            e2m1x8_to_h2(cw.y, h);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h[i]);
                out[4 + i] = __floats2bfloat162_rn(f.x * sf, f.y * sf);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) out[i] = __floats2bfloat162_rn(0.f, 0.f);
        }
        if (j < nsel) {
            uint4 *dst = reinterpret_cast<uint4 *>(krow + lane * 16);
            dst[0] = *reinterpret_cast<uint4 *>(&out[0]);
            dst[1] = *reinterpret_cast<uint4 *>(&out[4]);
            const __nv_bfloat162 r = s >= 0 ? reinterpret_cast<const __nv_bfloat162 *>(rope + size_t(s) * MLA_R)[lane]
                                            : __floats2bfloat162_rn(0.f, 0.f);
            reinterpret_cast<__nv_bfloat162 *>(krow + MLA_L)[lane] = r;
        }
        *reinterpret_cast<uint4 *>(&tile[jj][lane * 16]) = *reinterpret_cast<uint4 *>(&out[0]);
        *reinterpret_cast<uint4 *>(&tile[jj][lane * 16 + 8]) = *reinterpret_cast<uint4 *>(&out[4]);
    }
    __syncthreads();
    // Vt rows: dim d, keys j0..j0+31 (64 bytes): 4 threads per row, 16 bytes each
    const int nk = min(32, nsel - j0);
    for (int i = threadIdx.x; i < MLA_L * 4; i += blockDim.x) {
        const int d = i >> 2, part = i & 3;
        __nv_bfloat162 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __halves2bfloat162(tile[part * 8 + 2 * k][d], tile[part * 8 + 2 * k + 1][d]);
        if (part * 8 < nk)
            *reinterpret_cast<uint4 *>(Vt + (size_t(q) * MLA_L + d) * nsel + j0 + part * 8) =
                *reinterpret_cast<uint4 *>(v);
    }
}

// ------------------------------------------------------------------------------------------------ attend
struct MlaSmem {
    static constexpr int STAGE = 32 * 1024;   // S: Q k-block 16 KB + K k-block 16 KB; O: one Vt tile [256, 64] 32 KB
    static constexpr int P_BYTES = MLA_H * MLA_NB * 2;   // 32 KB: two swizzle atoms of [128 rows x 64 keys]
    static constexpr int BYTES = MLA_STAGES * STAGE + P_BYTES + 1024 + 1024;
};

__global__ void __launch_bounds__(MLA_THREADS, 1)
    mla_attend_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                      const __grid_constant__ CUtensorMap tma_v, const int32_t *__restrict__ idx, int nsel,
                      float scale_log2, float *__restrict__ part_o, float *__restrict__ part_ml, int *error) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ps = smem + MLA_STAGES * MlaSmem::STAGE;   // P, 1024-aligned
    uint64_t *full = reinterpret_cast<uint64_t *>(ps + MlaSmem::P_BYTES);
    uint64_t *empty = full + MLA_STAGES;
    uint64_t *sfull = empty + MLA_STAGES;
    uint64_t *pfull = sfull + 1;
    uint64_t *ofull = pfull + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ofull + 1);
    __shared__ int valid[MLA_NB];
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x, q = blockIdx.y;
    const int nblk = gridDim.x;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < MLA_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(sfull, 1);
        tc::mbar_init(pfull, 4);
        tc::mbar_init(ofull, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_q);
        tc::prefetch_tmap(&tma_k);
        tc::prefetch_tmap(&tma_v);
    }
    for (int j = threadIdx.x; j < MLA_NB; j += blockDim.x) {
        const int jj = blk * MLA_NB + j;
        valid[j] = jj < nsel && idx[size_t(q) * nsel + jj] >= 0;
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
        atomicExch(error, 1);
    };
    constexpr int KB_S = MLA_D / MLA_BK;   // 9 k-blocks of Q.K^T
    constexpr int KB_O = MLA_NB / MLA_BK;  // 2 k-blocks of P.V per half

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            auto next = [&]() {
                if (++stage == MLA_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            };
            for (int kb = 0; kb < KB_S && !abort_flag; ++kb, next()) {
                if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                    fail();
                    break;
                }
                uint8_t *sa = smem + stage * MlaSmem::STAGE;
                tc::mbar_arrive_expect_tx(&full[stage], 32 * 1024);
                tc::tma_load_2d(sa, &tma_q, &full[stage], kb * MLA_BK, q * MLA_H);
                tc::tma_load_2d(sa + 16 * 1024, &tma_k, &full[stage], kb * MLA_BK, q * nsel + blk * MLA_NB);
            }
            for (int half = 0; half < 2 && !abort_flag; ++half)
                for (int kb = 0; kb < KB_O && !abort_flag; ++kb, next()) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail();
                        break;
                    }
                    uint8_t *sa = smem + stage * MlaSmem::STAGE;
                    tc::mbar_arrive_expect_tx(&full[stage], 32 * 1024);
                    tc::tma_load_2d(sa, &tma_v, &full[stage], blk * MLA_NB + kb * MLA_BK, q * MLA_L + half * 256);
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            auto next = [&]() {
                if (++stage == MLA_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            };
            const uint32_t idesc_s = tc::idesc_bf16_f32(MLA_H, MLA_NB);
            const uint32_t idesc_o = tc::idesc_bf16_f32(MLA_H, 256);
            bool ok = true;
            for (int kb = 0; kb < KB_S && ok; ++kb, next()) {
                if (!(ok = tc::mbar_wait(&full[stage], phase))) break;
                tc::tc_fence_after();
                const uint32_t sa = tc::smem_u32(smem + stage * MlaSmem::STAGE);
                const uint64_t ad = tc::sw128_kmajor_desc(sa), bd = tc::sw128_kmajor_desc(sa + 16 * 1024);
#pragma unroll
                for (int k = 0; k < MLA_BK / 16; ++k)
                    tc::mma_f16(tmem + 256, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc_s,
                                (kb > 0 || k > 0) ? 1u : 0u);
                tc::mma_commit(&empty[stage]);
            }
            if (ok) tc::mma_commit(sfull);
            if (ok && !(ok = tc::mbar_wait(pfull, 0))) fail();
            tc::tc_fence_after();
            for (int half = 0; half < 2 && ok; ++half)
                for (int kb = 0; kb < KB_O && ok; ++kb, next()) {
                    if (!(ok = tc::mbar_wait(&full[stage], phase))) break;
                    tc::tc_fence_after();
                    const uint32_t sv = tc::smem_u32(smem + stage * MlaSmem::STAGE);
                    const uint64_t ad = tc::sw128_kmajor_desc(tc::smem_u32(ps) + kb * 16 * 1024);
                    const uint64_t bd = tc::sw128_kmajor_desc(sv);
#pragma unroll
                    for (int k = 0; k < MLA_BK / 16; ++k)
                        tc::mma_f16(tmem + uint32_t(half * 256), ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc_o,
                                    (kb > 0 || k > 0) ? 1u : 0u);
                    tc::mma_commit(&empty[stage]);
                }
            if (ok) tc::mma_commit(ofull);
            else fail();
        }
    } else {
        // softmax / epilogue: warp w reads TMEM lanes 32*(w%4)..+31 = heads
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;   // head
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        bool ok = true;
        if (lane == 0) ok = tc::mbar_wait(sfull, 0);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        float m = -INFINITY, l = 0.f;
        if (ok && !abort_flag) {
            tc::tc_fence_after();
            float sv[MLA_NB];
#pragma unroll
            for (int c = 0; c < MLA_NB / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(lane_base + 256 + uint32_t(c * 32), r);
                tc::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    sv[c * 32 + i] = valid[c * 32 + i] ? __uint_as_float(r[i]) * scale_log2 : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < MLA_NB; ++i) m = fmaxf(m, sv[i]);
            // P in BF16, 128-byte swizzled K-major: atom a = keys 64a..64a+63, row `row`, 16-byte chunk c at c ^ (row&7)
#pragma unroll
            for (int a = 0; a < 2; ++a) {
                uint8_t *rowp = ps + a * 16 * 1024 + row * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    __nv_bfloat162 pv[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int k0 = a * 64 + c * 8 + 2 * t;
                        const float p0 = m == -INFINITY ? 0.f : exp2f(sv[k0] - m);
                        const float p1 = m == -INFINITY ? 0.f : exp2f(sv[k0 + 1] - m);
                        pv[t] = __floats2bfloat162_rn(p0, p1);
                        const float2 back = __bfloat1622float2(pv[t]);
                        l += back.x + back.y;
                    }
                    *reinterpret_cast<uint4 *>(rowp + ((c ^ (row & 7)) << 4)) = *reinterpret_cast<uint4 *>(pv);
                }
            }
        }
        // P visible to the tensor core (async proxy), TMEM reads of S done before O overwrites it
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(pfull);
        if (lane == 0 && ok) ok = tc::mbar_wait(ofull, 0);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        const size_t unit = size_t(q) * nblk + blk;
        float *po = part_o + (unit * MLA_H + row) * MLA_L;
        if (ok && !abort_flag) {
            tc::tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < MLA_L / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(lane_base + uint32_t(c * 32), r);
                tc::tmem_ld_wait();
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    reinterpret_cast<float4 *>(po + c * 32)[v] =
                        make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            }
        } else {
            if (lane == 0 && !ok) fail();
            for (int c = 0; c < MLA_L; ++c) po[c] = 0.f;
            m = -INFINITY;
            l = 0.f;
        }
        part_ml[(unit * MLA_H + row) * 2] = m;
        part_ml[(unit * MLA_H + row) * 2 + 1] = l;
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------------ flash attention
// mla_flash: the selected keys of a query in one pass, online softmax, O accumulated in TMEM, FP16 operands. One CTA
// per (value half j, key split s, query q); 320 threads:
//   warp 0      MMA issuer (lane 0). Per 64-key block b: S = Q.K^T over the ring's five k-blocks (the other value
//               half and the rotary one) and this half's four (the V tile of b), then O += P.V of block b - 1 with P
//               read from TMEM and V read in place through an MN-major descriptor (no transposed copy)
//   warp 1      TMEM owner (512 columns: O half at 0..255, S buffers at 256 and 320, P buffers at 384 and 416)
//   warps 2-5   producers: TMA of the query's nine k-blocks once (converted to f16 by warps 2-9 together, below),
//               and the gather of every block's latent rows into
//               128-byte-swizzled K-major FP16 tiles (E2M1 -> f16 by the hardware conversion, times the block's E4M3
//               scale in f16: exact, every product has at most six significant bits and lies in f16's normal range;
//               the rotary part BF16 -> f16); a block's rows are loaded while the previous block is written, and the
//               slots one block further ahead
//   warps 6-9   softmax, one head row per thread: block max, lazy correction of O (only when
//               the running max grows by more than 2^8; then O and the row sum are rescaled in TMEM once P.V of the
//               previous block is done), P = 2^(S - m) in f16 into TMEM, the row sum over the rounded P, and the
//               epilogue (O / l, or the unnormalized split partial with m and l for mla_merge)
// The query is converted once, in place: each head row BF16 -> f16 scaled by the power of two 2^e that puts the row's
// largest magnitude in [2^14, 2^15) (exact down to 2^-28 of that magnitude); 2^-e is folded into the row's softmax
// scale. V is double-buffered, so S of block b does not wait for P.V of block b - 1: the tensor core computes S of b
// while the softmax warps work on b - 1. Every wait is bounded; a wait that runs out sets the error word, raises the
// CTA's abort flag and every role winds down (the output of that query is then meaningless and the caller raises).
constexpr int MF_NB = 64;
constexpr int MF_STAGES = 2;
constexpr int MF_THREADS = 320;
constexpr float MF_TAU = 8.f;      // log2 of the growth of the running max tolerated before O is rescaled
constexpr uint32_t MF_TS = 256;    // TMEM column of the S buffers (2 x 64)
constexpr uint32_t MF_TP = 384;    // TMEM column of the P buffers (2 x 32: 64 f16 per row)

struct MfSmem {
    static constexpr int QKB = MLA_H * 64 * 2;     // 16 KB: a query k-block [128 heads x 64 dims]
    static constexpr int Q = 9 * QKB;              // the whole query, resident
    static constexpr int KKB = MF_NB * 64 * 2;     // 8 KB: a key k-block [64 keys x 64 dims]
    static constexpr int VBUF = 4 * KKB;           // this value half's four k-blocks of one key block
    static constexpr int BYTES = Q + MF_STAGES * KKB + 2 * VBUF + 1024 + 1024;
};
static_assert(MfSmem::BYTES <= 232448, "mla_flash shared memory");

// k-block of ring position i (0..4): the other value half's four, then the rotary one
XT_DEV int mf_kb(int i, int j) { return i < 4 ? 4 * (1 - j) + i : 8; }

// 32 dims (four 16-byte chunks c0..c0+3 of a 128-byte swizzled row) of one NVFP4 latent k-block row -> f16
XT_DEV void mf_write_kb(uint8_t *rowp, int kk, int c0, const uint4 &cw, uint16_t sc) {
    const __half2 s2 = e4m3x2_to_h2(sc);
    const __half2 s0 = __low2half2(s2), s1 = __high2half2(s2);
    const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        __half2 hh[4];
        e2m1x8_to_h2(words[t], hh);
#pragma unroll
        for (int u = 0; u < 4; ++u) hh[u] = __hmul2(hh[u], t < 2 ? s0 : s1);
        *reinterpret_cast<uint4 *>(rowp + (((c0 + t) ^ (kk & 7)) << 4)) = *reinterpret_cast<uint4 *>(hh);
    }
}

// Largest magnitude of k-blocks [k0, k1) of query row `row` (BF16, 128 bytes per row and k-block)
XT_DEV float mf_row_amax(const uint8_t *qs, int row, int k0, int k1) {
    float a = 0.f;
    for (int kb = k0; kb < k1; ++kb) {
        const uint4 *p = reinterpret_cast<const uint4 *>(qs + kb * MfSmem::QKB + row * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {   // chunk order rotated by the row: the lanes of a warp hit distinct banks
            const uint4 v = p[c ^ (row & 7)];
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float2 f = __bfloat1622float2(h[u]);
                a = fmaxf(a, fmaxf(fabsf(f.x), fabsf(f.y)));
            }
        }
    }
    return a;
}

// The same k-blocks BF16 -> f16 in place, times qf (a power of two)
XT_DEV void mf_row_to_f16(uint8_t *qs, int row, int k0, int k1, float qf) {
    for (int kb = k0; kb < k1; ++kb) {
        uint4 *p = reinterpret_cast<uint4 *>(qs + kb * MfSmem::QKB + row * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 v = p[c ^ (row & 7)];
            auto cv = [qf](uint32_t w) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
                const __half2 hv = __floats2half2_rn(f.x * qf, f.y * qf);
                return *reinterpret_cast<const uint32_t *>(&hv);
            };
            p[c ^ (row & 7)] = make_uint4(cv(v.x), cv(v.y), cv(v.z), cv(v.w));
        }
    }
}

// 2^e with e chosen so that amax * 2^e lies in [2^14, 2^15) (1 for amax 0)
XT_DEV int mf_row_exp(float amax) {
    const int ex = int((__float_as_uint(amax) >> 23) & 0xFF);
    return amax > 0.f ? max(-126, min(126, 141 - ex)) : 0;
}

__global__ void __launch_bounds__(MF_THREADS, 1)
    mla_flash_kernel(const __grid_constant__ CUtensorMap tma_ql, const __grid_constant__ CUtensorMap tma_qr,
                     const int32_t *__restrict__ idx, int nsel, int bps, int nblk, const uint8_t *__restrict__ codes,
                     const uint8_t *__restrict__ scales, const __nv_bfloat16 *__restrict__ rope, float scale_log2,
                     __nv_bfloat16 *__restrict__ out, int64_t out_ts, int64_t out_hs, float *__restrict__ part_o,
                     float *__restrict__ part_ml, int nslots, int *error) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qs = smem;                                   // [9][128 x 64]
    uint8_t *ring = qs + MfSmem::Q;                       // [STAGES][64 x 64]
    uint8_t *vbuf = ring + MF_STAGES * MfSmem::KKB;       // [2][4][64 x 64]
    uint64_t *full = reinterpret_cast<uint64_t *>(vbuf + 2 * MfSmem::VBUF);
    uint64_t *empty = full + MF_STAGES;
    uint64_t *qfull = empty + MF_STAGES;
    uint64_t *qready = qfull + 1;
    uint64_t *vfull = qready + 1;          // [2]
    uint64_t *vfree = vfull + 2;           // [2]: P.V of the buffer's block done (V tile and P buffer free)
    uint64_t *sfull = vfree + 2;           // [2]
    uint64_t *sfree = sfull + 2;           // [2]
    uint64_t *pfull = sfree + 2;           // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pfull + 2);
    __shared__ volatile int abort_flag;
    // the query rows' largest magnitudes over k-blocks 0-4 and 5-8, exchanged once at the start in V tile 1 (first
    // written for block 1, which the MMA issuer starts only after every converting warp has arrived on qready)
    float (*row_amax)[MLA_H] = reinterpret_cast<float (*)[MLA_H]>(vbuf + MfSmem::VBUF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x, split = blockIdx.y, q = blockIdx.z, splits = gridDim.y;
    const int b0 = split * bps, b1 = min(nblk, b0 + bps), nb = b1 - b0;
    const int32_t *qidx = idx + size_t(q) * nsel;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < MF_STAGES; ++s) {
            tc::mbar_init(&full[s], 4);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(qfull, 1);
        tc::mbar_init(qready, 8);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&vfull[s], 4);
            tc::mbar_init(&vfree[s], 1);
            tc::mbar_init(&sfull[s], 1);
            tc::mbar_init(&sfree[s], 4);
            tc::mbar_init(&pfull[s], 4);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_ql);
        tc::prefetch_tmap(&tma_qr);
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
        atomicExch(error, 1);
    };
    // one lane waits, the warp follows; false once the wait ran out or another role failed
    auto warp_wait = [&](uint64_t *bar, uint32_t parity) {
        int good = 1;
        if (lane == 0) good = tc::mbar_wait(bar, parity);
        good = __shfl_sync(0xffffffffu, good, 0);
        return good && !abort_flag;
    };

    if (warp == 0) {
        if (lane == 0 && nb > 0) {
            int stage = 0;
            uint32_t phase = 0;
            const uint32_t idesc_s = tc::idesc_f16_f32(MLA_H, MF_NB);
            const uint32_t idesc_o = tc::idesc_f16_f32(MLA_H, 256) | (1u << 16);   // B (V) MN-major
            const uint32_t qa = tc::smem_u32(qs), va = tc::smem_u32(vbuf);
            bool ok = tc::mbar_wait(qready, 0);
            auto pv = [&](int b) {   // O (+)= P . V of block b; its completion frees the V tile and P buffer of b
                if (!(ok = tc::mbar_wait(&pfull[b & 1], uint32_t((b >> 1) & 1)))) return;
                tc::tc_fence_after();
                const uint32_t pa = tmem + MF_TP + uint32_t((b & 1) * 32);
                const uint32_t vb = va + uint32_t((b & 1) * MfSmem::VBUF);
#pragma unroll
                for (int k = 0; k < MF_NB / 16; ++k)
                    tc::mma_f16_ts(tmem, pa + uint32_t(8 * k),
                                   tc::sw128_mnmajor_desc(vb + uint32_t(k * 2048), MfSmem::KKB, 1024), idesc_o,
                                   (b > 0 || k > 0) ? 1u : 0u);
                tc::mma_commit(&vfree[b & 1]);
            };
            auto s_kb = [&](uint32_t sb, int kb, uint32_t baddr, bool first) {
                const uint64_t ad = tc::sw128_kmajor_desc(qa + uint32_t(kb * MfSmem::QKB));
                const uint64_t bd = tc::sw128_kmajor_desc(baddr);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    tc::mma_f16(sb, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc_s, (!first || k > 0) ? 1u : 0u);
            };
            for (int b = 0; b < nb && ok && !abort_flag; ++b) {
                const uint32_t sb = tmem + MF_TS + uint32_t((b & 1) * MF_NB);
                if (!(ok = tc::mbar_wait(&sfree[b & 1], uint32_t(((b >> 1) & 1) ^ 1)))) break;
                tc::tc_fence_after();
                for (int i = 0; i < 5 && ok; ++i) {   // the ring's k-blocks
                    if (!(ok = tc::mbar_wait(&full[stage], phase))) break;
                    tc::tc_fence_after();
                    s_kb(sb, mf_kb(i, j), tc::smem_u32(ring + stage * MfSmem::KKB), i == 0);
                    tc::mma_commit(&empty[stage]);
                    if (++stage == MF_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if (!(ok = tc::mbar_wait(&vfull[b & 1], uint32_t((b >> 1) & 1)))) break;
                tc::tc_fence_after();
                const uint32_t vb = va + uint32_t((b & 1) * MfSmem::VBUF);
#pragma unroll 1
                for (int t = 0; t < 4; ++t) s_kb(sb, 4 * j + t, vb + uint32_t(t * MfSmem::KKB), false);
                tc::mma_commit(&sfull[b & 1]);
                if (b > 0) pv(b - 1);
            }
            if (ok && !abort_flag) pv(nb - 1);
            if (!ok) fail();
        }
    } else if (warp >= 2 && warp < 6) {
        const int w = warp - 2;
        const int kk = w * 16 + (lane >> 1), half = lane & 1;   // key of the block, 32-dim half of a k-block
        if (w == 0 && lane == 0 && nb > 0) {   // the query, once: eight latent k-blocks and the rotary one
            tc::mbar_arrive_expect_tx(qfull, MfSmem::Q);
            for (int kb = 0; kb < 8; ++kb) tc::tma_load_3d(qs + kb * MfSmem::QKB, &tma_ql, qfull, kb * 64, q, 0);
            tc::tma_load_3d(qs + 8 * MfSmem::QKB, &tma_qr, qfull, 0, q, 0);
        }
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        uint4 ncw[8], nrp[4];
        uint32_t nsc[4];   // the E4M3 scale pairs of k-blocks r and r + 4 (low and high half)
        int pslot = nb > 0 ? qidx[size_t(b0) * MF_NB + kk] : -1;
        auto load_block = [&](int b) {   // this key's codes and scales of its half of every latent k-block (other
                                         // value half first), and its half of the rotary part
            int slot = pslot;
            if (nslots && slot >= nslots) {   // bounds-checked mode: skip the key, error word 2
                atomicCAS(error, 0, 2);
                slot = -1;
            }
            if (b + 1 < nb) pslot = qidx[size_t(b0 + b + 1) * MF_NB + kk];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const int kb = r < 4 ? 4 * (1 - j) + r : 4 * j + (r - 4);
                ncw[r] = slot >= 0 ? *reinterpret_cast<const uint4 *>(codes + size_t(slot) * (MLA_L / 2) + kb * 32 +
                                                                      half * 16)
                                   : make_uint4(0, 0, 0, 0);
            }
            // the key's 32 scales in two loads; this thread's pair of k-block kb is 16-bit half `half` of word kb
            uint4 sw[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
            if (slot >= 0) {
                sw[0] = reinterpret_cast<const uint4 *>(scales + size_t(slot) * (MLA_L / 16))[0];
                sw[1] = reinterpret_cast<const uint4 *>(scales + size_t(slot) * (MLA_L / 16))[1];
            }
            const uint32_t lo[4] = {sw[0].x, sw[0].y, sw[0].z, sw[0].w}, hi[4] = {sw[1].x, sw[1].y, sw[1].z, sw[1].w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {   // k-blocks 4 (1 - j) + r and 4 j + r
                const uint32_t a = j ? lo[r] : hi[r], c = j ? hi[r] : lo[r];
                nsc[r] = half ? __byte_perm(a, c, 0x7632) : __byte_perm(a, c, 0x5410);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t)
                nrp[t] = slot >= 0 ? reinterpret_cast<const uint4 *>(rope + size_t(slot) * MLA_R + half * 32)[t]
                                   : make_uint4(0, 0, 0, 0);
        };
        if (nb > 0) {
            load_block(0);
            // k-blocks 0-4 of the query row this thread shares with a softmax thread (which takes 5-8)
            const int qrow = (warp & 3) * 32 + lane;
            ok = warp_wait(qfull, 0);
            row_amax[0][qrow] = ok ? mf_row_amax(qs, qrow, 0, 5) : 0.f;
            asm volatile("bar.sync 1, 256;\n" ::: "memory");
            const int e = mf_row_exp(fmaxf(row_amax[0][qrow], row_amax[1][qrow]));
            if (ok) mf_row_to_f16(qs, qrow, 0, 5, __uint_as_float(uint32_t(127 + e) << 23));
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(qready);
        }
        for (int b = 0; b < nb && ok && !abort_flag; ++b) {
            uint4 cw[8], rp[4];
            uint16_t sc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                cw[i] = ncw[i];
                sc[i] = uint16_t(nsc[i & 3] >> (i < 4 ? 0 : 16));
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) rp[t] = nrp[t];
            if (b + 1 < nb) load_block(b + 1);
            // the ring: the other value half's four k-blocks, then the rotary one
#pragma unroll
            for (int i = 0; i < 5; ++i) {
                if (!(ok = warp_wait(&empty[stage], phase ^ 1))) break;
                uint8_t *rowp = ring + stage * MfSmem::KKB + kk * 128;
                if (i < 4) {
                    mf_write_kb(rowp, kk, half * 4, cw[i], sc[i]);
                } else {
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const __nv_bfloat162 *bp = reinterpret_cast<const __nv_bfloat162 *>(&rp[t]);
                        __half2 hh[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) hh[u] = __float22half2_rn(__bfloat1622float2(bp[u]));
                        const int c = half * 4 + t;
                        *reinterpret_cast<uint4 *>(rowp + ((c ^ (kk & 7)) << 4)) = *reinterpret_cast<uint4 *>(hh);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&full[stage]);
                if (++stage == MF_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            // this half's four k-blocks into V tile b & 1, once P.V of block b - 2 has read it
            if (b >= 2 && !(ok = warp_wait(&vfree[b & 1], uint32_t(((b >> 1) & 1) ^ 1)))) break;
            uint8_t *vrow = vbuf + (b & 1) * MfSmem::VBUF + kk * 128;
#pragma unroll
            for (int t = 0; t < 4; ++t) mf_write_kb(vrow + t * MfSmem::KKB, kk, half * 4, cw[4 + t], sc[4 + t]);
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&vfull[b & 1]);
        }
        if (!ok && lane == 0) fail();
    } else if (warp >= 6) {
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;   // head
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        float m = -INFINITY, l = 0.f, sl = scale_log2;
        bool ok = true;
        if (nb > 0) {   // k-blocks 5-8 of this head row of the query (a producer thread takes 0-4)
            ok = warp_wait(qfull, 0);
            row_amax[1][row] = ok ? mf_row_amax(qs, row, 5, 9) : 0.f;
            asm volatile("bar.sync 1, 256;\n" ::: "memory");
            const int e = mf_row_exp(fmaxf(row_amax[0][row], row_amax[1][row]));
            if (ok) mf_row_to_f16(qs, row, 5, 9, __uint_as_float(uint32_t(127 + e) << 23));
            sl = scale_log2 * __uint_as_float(uint32_t(127 - e) << 23);
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(qready);
        }
        int ilo = nb > 0 ? qidx[size_t(b0) * MF_NB + lane] : -1;
        int ihi = nb > 0 ? qidx[size_t(b0) * MF_NB + 32 + lane] : -1;
        for (int b = 0; b < nb && ok; ++b) {
            if (!(ok = warp_wait(&sfull[b & 1], uint32_t((b >> 1) & 1)))) break;
            tc::tc_fence_after();
            float sv[MF_NB];
#pragma unroll
            for (int c = 0; c < MF_NB / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(lane_base + MF_TS + uint32_t((b & 1) * MF_NB + c * 32), r);
                tc::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(r[i]);
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&sfree[b & 1]);
            // keys with a slot, and in bounds-checked mode only slots inside the cache (the producers skip the rest)
            const unsigned vlo = __ballot_sync(0xffffffffu, ilo >= 0 && (!nslots || ilo < nslots));
            const unsigned vhi = __ballot_sync(0xffffffffu, ihi >= 0 && (!nslots || ihi < nslots));
            if (b + 1 < nb) {   // the next block's slots, in flight while this block is processed
                ilo = qidx[size_t(b0 + b + 1) * MF_NB + lane];
                ihi = qidx[size_t(b0 + b + 1) * MF_NB + 32 + lane];
            }
            float bm = -INFINITY;
#pragma unroll
            for (int i = 0; i < MF_NB; ++i) {
                const bool v = i < 32 ? (vlo >> i) & 1 : (vhi >> (i - 32)) & 1;
                sv[i] = v ? sv[i] * sl : -INFINITY;
                bm = fmaxf(bm, sv[i]);
            }
            const float m_new = fmaxf(m, bm);
            const bool need = m_new > -INFINITY && (m == -INFINITY || m_new > m + MF_TAU);
            float factor = 1.f;
            if (need) {
                factor = m == -INFINITY ? 0.f : ex2_approx(m - m_new);
                m = m_new;
                l *= factor;
            }
            if (b > 0 && __ballot_sync(0xffffffffu, need)) {   // O complete up to block b - 1, then rescaled
                if (!(ok = warp_wait(&vfree[(b - 1) & 1], uint32_t(((b - 1) >> 1) & 1)))) break;
                tc::tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t r[32];
                    tc::tmem_ld32(lane_base + uint32_t(c * 32), r);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
                    tc::tmem_st32(lane_base + uint32_t(c * 32), r);
                }
                tc::tmem_st_wait();
            }
            uint32_t pr[32];
            float lacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float p0 = m == -INFINITY ? 0.f : ex2_approx(sv[2 * c] - m);
                const float p1 = m == -INFINITY ? 0.f : ex2_approx(sv[2 * c + 1] - m);
                const __half2 h = __floats2half2_rn(p0, p1);
                const float2 back = __half22float2(h);
                lacc[c & 3] += back.x + back.y;
                pr[c] = *reinterpret_cast<const uint32_t *>(&h);
            }
            l += (lacc[0] + lacc[1]) + (lacc[2] + lacc[3]);
            // P buffer b & 1 was last read by P.V of block b - 2
            if (b >= 2 && !(ok = warp_wait(&vfree[b & 1], uint32_t(((b >> 1) & 1) ^ 1)))) break;
            tc::tc_fence_after();
            tc::tmem_st32(lane_base + MF_TP + uint32_t((b & 1) * 32), pr);
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&pfull[b & 1]);
        }
        int good = ok ? 1 : 0;
        if (ok && nb > 0 && lane == 0) good = tc::mbar_wait(&vfree[(nb - 1) & 1], uint32_t(((nb - 1) >> 1) & 1));
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good && lane == 0) fail();
        tc::tc_fence_after();
        const size_t pbase = (size_t(q) * splits + split) * MLA_H + row;
        if (good && nb > 0 && !abort_flag) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(lane_base + uint32_t(c * 32), r);
                tc::tmem_ld_wait();
                if (splits == 1) {
                    __nv_bfloat16 *dst = out + q * out_ts + row * out_hs + j * 256 + c * 32;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        __nv_bfloat162 o[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            o[u] = __floats2bfloat162_rn(__uint_as_float(r[8 * v + 2 * u]) * inv,
                                                         __uint_as_float(r[8 * v + 2 * u + 1]) * inv);
                        reinterpret_cast<uint4 *>(dst)[v] = *reinterpret_cast<uint4 *>(o);
                    }
                } else {
                    float *dst = part_o + pbase * MLA_L + j * 256 + c * 32;
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        reinterpret_cast<float4 *>(dst)[v] =
                            make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                        __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                }
            }
        } else if (splits > 1) {
            for (int c = 0; c < 256; ++c) part_o[pbase * MLA_L + j * 256 + c] = 0.f;
            m = -INFINITY;
            l = 0.f;
        }
        if (splits > 1 && j == 0) {
            part_ml[pbase * 2] = (good && nb > 0) ? m : -INFINITY;
            part_ml[pbase * 2 + 1] = (good && nb > 0) ? l : 0.f;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------------ merge
// grid (heads, queries), 128 threads: thread t -> dims 4t..4t+3
__global__ void __launch_bounds__(128) mla_merge_kernel(const float *__restrict__ part_o,
                                                        const float *__restrict__ part_ml, int nblk,
                                                        __nv_bfloat16 *__restrict__ out) {
    const int h = blockIdx.x, q = blockIdx.y;
    float M = -INFINITY;
    for (int b = 0; b < nblk; ++b) M = fmaxf(M, part_ml[((size_t(q) * nblk + b) * MLA_H + h) * 2]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b < nblk; ++b) {
        const size_t unit = (size_t(q) * nblk + b) * MLA_H + h;
        const float mb = part_ml[unit * 2];
        const float f = mb == -INFINITY ? 0.f : exp2f(mb - M);
        L += part_ml[unit * 2 + 1] * f;
        const float4 v = reinterpret_cast<const float4 *>(part_o + unit * MLA_L)[threadIdx.x];
        o.x += v.x * f;
        o.y += v.y * f;
        o.z += v.z * f;
        o.w += v.w * f;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    __nv_bfloat162 *dst = reinterpret_cast<__nv_bfloat162 *>(out + (size_t(q) * MLA_H + h) * MLA_L) + threadIdx.x * 2;
    dst[0] = __floats2bfloat162_rn(o.x * inv, o.y * inv);
    dst[1] = __floats2bfloat162_rn(o.z * inv, o.w * inv);
}

}  // namespace xt

using namespace xt;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 mla_encode_fn() {
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

bool mla_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = mla_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
    cuuint32_t box[2] = {cuuint32_t(MLA_BK), box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [Q, 128 heads, d] BF16 view (unit stride along d, element strides ts, hs) as a 3-D map (d, Q, heads) whose box is
// one query's 128 heads x 64 values: a 128-row 128-byte-swizzled tile
bool mla_map3(CUtensorMap *map, const void *ptr, int d, int Q, int64_t ts, int64_t hs) {
    auto fn = mla_encode_fn();
    if (!fn || ts <= 0 || hs <= 0 || (ts * 2) % 16 || (hs * 2) % 16 || reinterpret_cast<uintptr_t>(ptr) % 16)
        return false;
    cuuint64_t dims[3] = {cuuint64_t(d), cuuint64_t(Q), cuuint64_t(MLA_H)};
    cuuint64_t strides[2] = {cuuint64_t(ts) * 2, cuuint64_t(hs) * 2};
    cuuint32_t box[3] = {64, 1, MLA_H};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" {

// lat [T, 576] bf16 -> cache slot[t] (codes [slots, 256] u8, scales [slots, 32] u8, rope [slots, 64] bf16)
int xt_mla_kv_write(const void *lat, const int64_t *slot, void *codes, void *scales, void *rope, int T,
                    cudaStream_t stream) {
    if (T <= 0) return 0;
    const int warps = 8;
    mla_kv_write_kernel<<<(T + warps - 1) / warps, warps * 32, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(lat), slot, static_cast<uint8_t *>(codes), static_cast<uint8_t *>(scales),
        static_cast<__nv_bfloat16 *>(rope), T);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Attention of Q queries (128 heads each) over their selected cache slots. q [Q, 128, 576] bf16 (absorbed: latent
// part q_nope . W_uk, then the rotary part), idx [Q, nsel] int32 (nsel % 128 == 0; -1 = no key), scratch: Kg [Q, nsel,
// 576] bf16, Vt [Q, 512, nsel] bf16, part_o [Q, nsel/128, 128, 512] f32, part_ml [Q, nsel/128, 128, 2] f32.
// out [Q, 128, 512] bf16 = softmax(scale * q.k) . v over the selected keys (latent values).
int xt_mla_decode(const void *q, const int32_t *idx, int Q, int nsel, const void *codes, const void *scales,
                  const void *rope, void *Kg, void *Vt, float *part_o, float *part_ml, void *out, float scale,
                  int *error, cudaStream_t stream) {
    if (Q <= 0 || nsel <= 0 || nsel % MLA_NB) return -2;
    dim3 gg(nsel / 32, Q);
    mla_gather_kernel<<<gg, 256, 0, stream>>>(idx, nsel, static_cast<const uint8_t *>(codes),
                                              static_cast<const uint8_t *>(scales),
                                              static_cast<const __nv_bfloat16 *>(rope),
                                              static_cast<__nv_bfloat16 *>(Kg), static_cast<__nv_bfloat16 *>(Vt));
    if (cudaGetLastError() != cudaSuccess) return -1;
    CUtensorMap mq, mk, mv;
    if (!mla_map(&mq, q, uint64_t(Q) * MLA_H, MLA_D, MLA_H) ||
        !mla_map(&mk, Kg, uint64_t(Q) * nsel, MLA_D, MLA_NB) ||
        !mla_map(&mv, Vt, uint64_t(Q) * MLA_L, uint64_t(nsel), 256))
        return -3;
    if (xt_smem_optin(mla_attend_kernel, int(MlaSmem::BYTES)) != cudaSuccess) return -4;
    const int nblk = nsel / MLA_NB;
    dim3 ga(nblk, Q);
    mla_attend_kernel<<<ga, MLA_THREADS, MlaSmem::BYTES, stream>>>(mq, mk, mv, idx, nsel,
                                                                  scale * 1.4426950408889634f, part_o, part_ml, error);
    if (cudaGetLastError() != cudaSuccess) return -1;
    dim3 gm(MLA_H, Q);
    mla_merge_kernel<<<gm, 128, 0, stream>>>(part_o, part_ml, nblk, static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Flash form of xt_mla_decode without gather scratch. The query comes as two views of [Q, 128 heads, d] BF16 with
// unit stride along d and element strides (token, head): the latent part q_lat (d = 512) and the rotary part q_rope
// (d = 64); out [Q, 128, 512] BF16 likewise (token and head strides out_ts, out_hs). part_o [Q, splits, 128, 512] f32
// and part_ml [Q, splits, 128, 2] are used only when splits > 1 (the splits' partials, merged by mla_merge, which
// writes a contiguous out). nsel % 64 == 0. nslots > 0 checks every selected slot against the cache size (a slot at or
// past it is skipped and sets the error word to 2); 0 skips the check.
int xt_mla_flash(const void *q_lat, int64_t ql_ts, int64_t ql_hs, const void *q_rope, int64_t qr_ts, int64_t qr_hs,
                 const int32_t *idx, int Q, int nsel, const void *codes, const void *scales, const void *rope,
                 float *part_o, float *part_ml, void *out, int64_t out_ts, int64_t out_hs, float scale, int splits,
                 int nslots, int *error, cudaStream_t stream) {
    if (Q <= 0 || Q > 65535 || nsel <= 0 || nsel % MF_NB || splits < 1 || nslots < 0) return -2;
    const int nblk = nsel / MF_NB;
    const int bps = (nblk + splits - 1) / splits;
    splits = (nblk + bps - 1) / bps;
    if (splits > 1 && (!part_o || !part_ml)) return -2;
    if (splits > 1 && (out_ts != int64_t(MLA_H) * MLA_L || out_hs != MLA_L)) return -2;
    if ((out_ts | out_hs) % 8 || reinterpret_cast<uintptr_t>(out) % 16) return -2;
    CUtensorMap ml, mr;
    if (!mla_map3(&ml, q_lat, MLA_L, Q, ql_ts, ql_hs) || !mla_map3(&mr, q_rope, MLA_R, Q, qr_ts, qr_hs)) return -3;
    if (xt_smem_optin(mla_flash_kernel, int(MfSmem::BYTES)) != cudaSuccess) return -4;
    mla_flash_kernel<<<dim3(2, splits, Q), MF_THREADS, MfSmem::BYTES, stream>>>(
        ml, mr, idx, nsel, bps, nblk, static_cast<const uint8_t *>(codes), static_cast<const uint8_t *>(scales),
        static_cast<const __nv_bfloat16 *>(rope), scale * 1.4426950408889634f, static_cast<__nv_bfloat16 *>(out),
        out_ts, out_hs, part_o, part_ml, nslots, error);
    if (cudaGetLastError() != cudaSuccess) return -1;
    if (splits > 1) {
        mla_merge_kernel<<<dim3(MLA_H, Q), 128, 0, stream>>>(part_o, part_ml, splits,
                                                             static_cast<__nv_bfloat16 *>(out));
        if (cudaGetLastError() != cudaSuccess) return -1;
    }
    return 0;
}

}  // extern "C"
