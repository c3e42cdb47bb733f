// Causal GQA prefill attention on the tcgen05 tensor cores (BF16 in, FP32 accumulate, head dim 128).
//
// out[t, h] = softmax(scale * q[t, h] . K[g]^T) . V[g] over the keys 0 .. start + t of kv head g = h / (Hq / Hkv), where
// query t sits at position start + t (a first chunk has start 0; a continuation chunk sees the whole cache before it).
// One CTA per (pair of 128-query tiles, query head), heaviest tiles first; 384 threads (three warpgroups):
//   warp 0      TMA producer (lane 0): the two query tiles once, then per 128-key tile j its K tile and V tile (two
//               2-stage rings) from the [rows, 128] BF16 cache, 128-byte swizzled
//   warp 1      TMEM owner (512 columns: S0 0..127, S1 128..255, O0 256..383, O1 384..511) and MMA issuer (lane 0):
//               S_t = Q_t . K_j^T, and O_t += P_t . V_j with P read from TMEM (it overwrites the first 64 columns of
//               S_t) and V through an MN-major descriptor (read in place, no transposed copy). The issue order
//               PV0_j, QK0_j+1, PV1_j, QK1_j+1 lets each softmax group work on one tile while the tensor core runs the
//               other tile's two products
//   warps 2-3   idle (they fill the first warpgroup)
//   warps 4-7   softmax of tile 0, one query row per thread (its TMEM lane); warps 8-11 the same for tile 1. Per key
//               tile: the row's 128 scores, the causal mask on the tiles that cross the diagonal, the running max with
//               a lazy correction (O and the row sum are rescaled only when the max grows by more than 2^8, once P.V
//               of the previous tile is done), P = 2^(s * scale * log2 e - m) in BF16 into TMEM; at the end O / l in
//               BF16 to the output rows
// Every wait is bounded: a wait that runs out sets the error word, raises the CTA's abort flag and every role winds
// down (the output is then meaningless and the caller raises). Reference parity: the reference runs prefill attention
// through its serving engine's library kernels (SGLang's FlashInfer / FA backends behind xtier/backend/method.py); this
// kernel is the B200-native replacement of that path.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "params.h"
#include "tc_common.cuh"

namespace xt {

constexpr int AP_BM = 128;            // query rows per tile (two tiles per CTA)
constexpr int AP_BN = 128;            // keys per tile
constexpr int AP_D = 128;             // head dim
constexpr int AP_KS = 2;              // K ring stages
constexpr int AP_VS = 2;              // V ring stages
constexpr int AP_THREADS = 384;
constexpr float AP_TAU = 8.f;         // log2 of the running-max growth tolerated before O is rescaled
constexpr int AP_REG_LAUNCH = 168;    // registers per thread at launch (65536 / 384, rounded to the allocation unit)
constexpr int AP_REG_LOW = 72;        // first warpgroup after the split
constexpr int AP_REG_HIGH = 216;      // softmax warpgroups after the split
static_assert(128 * AP_REG_LOW + 256 * AP_REG_HIGH <= AP_THREADS * AP_REG_LAUNCH, "register split over budget");

struct ApSmem {
    static constexpr int PANEL = 128 * 128;          // 16 KB: 128 rows x 64 BF16 (one 128-byte swizzled panel)
    static constexpr int TILE = 2 * PANEL;           // 32 KB: 128 rows x 128 dims
    static constexpr int Q = 2 * TILE;               // the CTA's two query tiles
    static constexpr int K = AP_KS * TILE;
    static constexpr int V = AP_VS * TILE;
    static constexpr int BYTES = Q + K + V + 256 + 1024;
};
static_assert(ApSmem::BYTES <= 232448, "attn_prefill shared memory");

// Number of 128-key tiles query tile `t` of the CTA at q0 needs (keys up to its last valid row's position)
XT_DEV int ap_key_tiles(int start, int q0, int t, int T) {
    const int last = min(start + q0 + AP_BM * t + AP_BM - 1, start + T - 1);
    return last / AP_BN + 1;
}

// The 128 FP32 columns of this thread's TMEM lane starting at `taddr`, waited for inside the same statement (no use of
// the registers can be scheduled before the wait).
XT_DEV void ap_ld128(uint32_t taddr, float (&v)[128]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
        "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, "
        "%22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, "
        "%42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, "
        "%62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, "
        "%82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, "
        "%101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, "
        "%117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127"
        "}, [%128];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
          "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15]),
          "=f"(v[16]), "=f"(v[17]), "=f"(v[18]), "=f"(v[19]), "=f"(v[20]), "=f"(v[21]), "=f"(v[22]), "=f"(v[23]),
          "=f"(v[24]), "=f"(v[25]), "=f"(v[26]), "=f"(v[27]), "=f"(v[28]), "=f"(v[29]), "=f"(v[30]), "=f"(v[31]),
          "=f"(v[32]), "=f"(v[33]), "=f"(v[34]), "=f"(v[35]), "=f"(v[36]), "=f"(v[37]), "=f"(v[38]), "=f"(v[39]),
          "=f"(v[40]), "=f"(v[41]), "=f"(v[42]), "=f"(v[43]), "=f"(v[44]), "=f"(v[45]), "=f"(v[46]), "=f"(v[47]),
          "=f"(v[48]), "=f"(v[49]), "=f"(v[50]), "=f"(v[51]), "=f"(v[52]), "=f"(v[53]), "=f"(v[54]), "=f"(v[55]),
          "=f"(v[56]), "=f"(v[57]), "=f"(v[58]), "=f"(v[59]), "=f"(v[60]), "=f"(v[61]), "=f"(v[62]), "=f"(v[63]),
          "=f"(v[64]), "=f"(v[65]), "=f"(v[66]), "=f"(v[67]), "=f"(v[68]), "=f"(v[69]), "=f"(v[70]), "=f"(v[71]),
          "=f"(v[72]), "=f"(v[73]), "=f"(v[74]), "=f"(v[75]), "=f"(v[76]), "=f"(v[77]), "=f"(v[78]), "=f"(v[79]),
          "=f"(v[80]), "=f"(v[81]), "=f"(v[82]), "=f"(v[83]), "=f"(v[84]), "=f"(v[85]), "=f"(v[86]), "=f"(v[87]),
          "=f"(v[88]), "=f"(v[89]), "=f"(v[90]), "=f"(v[91]), "=f"(v[92]), "=f"(v[93]), "=f"(v[94]), "=f"(v[95]),
          "=f"(v[96]), "=f"(v[97]), "=f"(v[98]), "=f"(v[99]), "=f"(v[100]), "=f"(v[101]), "=f"(v[102]),
          "=f"(v[103]), "=f"(v[104]), "=f"(v[105]), "=f"(v[106]), "=f"(v[107]), "=f"(v[108]), "=f"(v[109]),
          "=f"(v[110]), "=f"(v[111]), "=f"(v[112]), "=f"(v[113]), "=f"(v[114]), "=f"(v[115]), "=f"(v[116]),
          "=f"(v[117]), "=f"(v[118]), "=f"(v[119]), "=f"(v[120]), "=f"(v[121]), "=f"(v[122]), "=f"(v[123]),
          "=f"(v[124]), "=f"(v[125]), "=f"(v[126]), "=f"(v[127])
        : "r"(taddr)
        : "memory");
}

// ---- packed FP32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes' worth of FMA / add)
XT_DEV uint64_t ap_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
XT_DEV void ap_unpack(uint64_t v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
XT_DEV uint64_t ap_fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
XT_DEV uint64_t ap_add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
XT_DEV float ap_max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^x for a pair on the FMA pipe (part of the exponentials move off the MUFU unit, which one softmax row per
// thread otherwise saturates): x = j + f with j = round(x) by the 1.5 * 2^23 addition (round-to-nearest), 2^f on
// [-1/2, 1/2] by a degree-3 polynomial (coefficients fitted here by reweighted least squares for relative error;
// max 1.1e-4, below BF16's 2^-9), and 2^j added to the exponent field. x is clamped at -125 (2^-125 for a masked key
// is 0 for every later use: the BF16 P times V and the row sum).
constexpr int AP_EMU = 0;   // default: pairs of every 8 whose exponentials take the polynomial (measured best: none)
XT_DEV void ap_exp2_poly(float x0, float x1, float &p0, float &p1) {
    const uint64_t magic = ap_pack(12582912.f, 12582912.f), nmagic = ap_pack(-12582912.f, -12582912.f);
    const uint64_t neg1 = ap_pack(-1.f, -1.f);
    const uint64_t c0 = ap_pack(0.99994045f, 0.99994045f), c1 = ap_pack(0.69341046f, 0.69341046f);
    const uint64_t c2 = ap_pack(0.24250269f, 0.24250269f), c3 = ap_pack(0.05432819f, 0.05432819f);
    const uint64_t xx = ap_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
    const uint64_t t = ap_add2(xx, magic);
    const uint64_t f = ap_fma2(ap_add2(t, nmagic), neg1, xx);
    uint64_t q = ap_fma2(c3, f, c2);
    q = ap_fma2(q, f, c1);
    q = ap_fma2(q, f, c0);
    float q0, q1, t0, t1;
    ap_unpack(q, q0, q1);
    ap_unpack(t, t0, t1);
    p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
    p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// 2^x for a pair through one packed half-precision MUFU operation (two exponentials per instruction): x rounded to
// f16 (relative 2^-11; the scores that matter lie in [-16, 8], so the absolute error of x stays below 2^-7 and that of
// 2^x below 0.6 % only where 2^x < 2^-8), the result widened back to FP32 for the BF16 P and the FP32 row sum.
constexpr int AP_EXP_H2 = 9;
XT_DEV void ap_exp2_h2(float x0, float x1, float &p0, float &p1) {
    uint32_t h, e;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(x1), "f"(x0));
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(h));
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&e));
    p0 = f.x;
    p1 = f.y;
}

template <int EMU>
__global__ void __launch_bounds__(AP_THREADS, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                        const __grid_constant__ CUtensorMap tma_v, int T, int start, int Hq, int group, int kv_row0,
                        int kv_hs, float scale_log2, __nv_bfloat16 *__restrict__ out, int64_t out_ts, int64_t out_hs,
                        const unsigned long long *__restrict__ tree, int *error) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qs = smem;                         // [2 tiles][2 panels][128 x 64]
    uint8_t *ks = qs + ApSmem::Q;               // [KS][2 panels][128 x 64]
    uint8_t *vs = ks + ApSmem::K;               // [VS][2 panels][128 x 64]
    uint64_t *bars = reinterpret_cast<uint64_t *>(vs + ApSmem::V);
    uint64_t *qfull = bars;                     // [1]
    uint64_t *kfull = qfull + 1;                // [KS]
    uint64_t *kfree = kfull + AP_KS;            // [KS]
    uint64_t *vfull = kfree + AP_KS;            // [VS]
    uint64_t *vfree = vfull + AP_VS;            // [VS]
    uint64_t *sfull = vfree + AP_VS;            // [2 tiles]
    uint64_t *pfull = sfull + 2;                // [2 tiles]: P of the tile written (4 softmax warps)
    uint64_t *pvdone = pfull + 2;               // [2 tiles]: P.V of the tile's latest key tile done
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pvdone + 2);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (T + 2 * AP_BM - 1) / (2 * AP_BM);
    const int qt = nqt - 1 - int(blockIdx.x) / Hq;   // heaviest (latest) query tiles first
    const int h = int(blockIdx.x) % Hq;
    const int g = h / group;
    const int q0 = qt * 2 * AP_BM;
    const int nk0 = ap_key_tiles(start, q0, 0, T), nk1 = ap_key_tiles(start, q0, 1, T);
    const int krow = kv_row0 + g * kv_hs;       // cache row of key 0 of this kv head
    if (threadIdx.x == 0) {
        abort_flag = 0;
        tc::mbar_init(qfull, 1);
        for (int s = 0; s < AP_KS; ++s) {
            tc::mbar_init(&kfull[s], 1);
            tc::mbar_init(&kfree[s], 1);
        }
        for (int s = 0; s < AP_VS; ++s) {
            tc::mbar_init(&vfull[s], 1);
            tc::mbar_init(&vfree[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            tc::mbar_init(&sfull[t], 1);
            tc::mbar_init(&pfull[t], 4);
            tc::mbar_init(&pvdone[t], 1);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tma_q);
        tc::prefetch_tmap(&tma_k);
        tc::prefetch_tmap(&tma_v);
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

    // register split: the first warpgroup (TMA, MMA, idle) gives registers to the two softmax warpgroups. The sum
    // 128 x AP_REG_LOW + 256 x AP_REG_HIGH equals the 384 x AP_REG_LAUNCH the block is launched with; the host checks
    // the launch count before the first launch (a split above it would wait forever)
    if (warp == 0) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(AP_REG_LOW));
        if (lane == 0) {
            bool ok = true;
            tc::mbar_arrive_expect_tx(qfull, ApSmem::Q);
            for (int t = 0; t < 2; ++t)
                for (int p = 0; p < 2; ++p)
                    tc::tma_load_3d(qs + t * ApSmem::TILE + p * ApSmem::PANEL, &tma_q, qfull, p * 64, h,
                                    q0 + t * AP_BM);
            // key order, K before V: the MMA issuer frees a K stage (both tiles' S) before the V stage of the same
            // key tile (both tiles' P.V), so this order never waits on a V stage while a K stage could be loaded
            for (int j = 0; j < nk1 && ok && !abort_flag; ++j) {
                const int sk = j % AP_KS, sv = j % AP_VS;
                if (j >= AP_KS && !(ok = tc::mbar_wait(&kfree[sk], uint32_t(((j / AP_KS) & 1) ^ 1)))) break;
                tc::mbar_arrive_expect_tx(&kfull[sk], ApSmem::TILE);
                for (int p = 0; p < 2; ++p)
                    tc::tma_load_2d(ks + sk * ApSmem::TILE + p * ApSmem::PANEL, &tma_k, &kfull[sk], p * 64,
                                    krow + j * AP_BN);
                if (j >= AP_VS && !(ok = tc::mbar_wait(&vfree[sv], uint32_t(((j / AP_VS) & 1) ^ 1)))) break;
                tc::mbar_arrive_expect_tx(&vfull[sv], ApSmem::TILE);
                for (int p = 0; p < 2; ++p)
                    tc::tma_load_2d(vs + sv * ApSmem::TILE + p * ApSmem::PANEL, &tma_v, &vfull[sv], p * 64,
                                    krow + j * AP_BN);
            }
            if (!ok) fail();
        }
    } else if (warp == 1) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(AP_REG_LOW));
        if (lane == 0) {
            bool ok = tc::mbar_wait(qfull, 0);
            const uint32_t idesc_s = tc::idesc_bf16_f32(AP_BM, AP_BN);
            const uint32_t idesc_o = tc::idesc_bf16_f32(AP_BM, AP_D) | (1u << 16);   // B (V) MN-major
            const uint32_t qa = tc::smem_u32(qs), ka = tc::smem_u32(ks), va = tc::smem_u32(vs);
            auto qk = [&](int t, int j) {   // S_t = Q_t . K_j^T
                const int s = j % AP_KS;
                if (!ok || !(ok = tc::mbar_wait(&kfull[s], uint32_t((j / AP_KS) & 1)))) return;
                tc::tc_fence_after();
                const uint32_t qb = qa + uint32_t(t * ApSmem::TILE), kb = ka + uint32_t(s * ApSmem::TILE);
#pragma unroll
                for (int k = 0; k < AP_D / 16; ++k) {
                    const uint32_t off = uint32_t((k >> 2) * ApSmem::PANEL + (k & 3) * 32);
                    tc::mma_f16(tmem + uint32_t(t * 128), tc::sw128_kmajor_desc(qb + off),
                                tc::sw128_kmajor_desc(kb + off), idesc_s, k > 0 ? 1u : 0u);
                }
                tc::mma_commit(&sfull[t]);
            };
            auto pv = [&](int t, int j) {   // O_t (+)= P_t . V_j
                const int s = j % AP_VS;
                if (!ok || !(ok = tc::mbar_wait(&pfull[t], uint32_t(j & 1)))) return;
                if (!(ok = tc::mbar_wait(&vfull[s], uint32_t((j / AP_VS) & 1)))) return;
                tc::tc_fence_after();
                const uint32_t vb = va + uint32_t(s * ApSmem::TILE);
                const uint32_t pt = tmem + uint32_t(t * 128), ot = tmem + 256u + uint32_t(t * 128);
#pragma unroll
                for (int k = 0; k < AP_BN / 16; ++k)
                    tc::mma_f16_ts(ot, pt + uint32_t(8 * k),
                                   tc::sw128_mnmajor_desc(vb + uint32_t(k * 2048), ApSmem::PANEL, 1024), idesc_o,
                                   (j > 0 || k > 0) ? 1u : 0u);
                tc::mma_commit(&pvdone[t]);
            };
            qk(0, 0);
            qk(1, 0);
            if (ok) tc::mma_commit(&kfree[0]);
            for (int j = 0; j < nk1 && ok && !abort_flag; ++j) {
                if (j < nk0) pv(0, j);
                if (j + 1 < nk0) qk(0, j + 1);
                pv(1, j);
                if (ok) tc::mma_commit(&vfree[j % AP_VS]);
                if (j + 1 < nk1) {
                    qk(1, j + 1);
                    if (ok) tc::mma_commit(&kfree[(j + 1) % AP_KS]);
                }
            }
            if (!ok) fail();
        }
    } else if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(AP_REG_LOW));
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(AP_REG_HIGH));
        const int t = warp < 8 ? 0 : 1;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;   // TMEM lane = query row of the tile
        const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
        const uint32_t st = lane_base + uint32_t(t * 128), ot = lane_base + 256u + uint32_t(t * 128);
        const int nk = t ? nk1 : nk0;
        const int qmin = start + q0 + t * AP_BM;   // position of the tile's first row
        const int qpos = qmin + row;
        // tree drafts: row r sees the keys before `start` and the tree keys (slots start + i) whose bit i is set
        const int trow = q0 + t * AP_BM + row;
        const unsigned long long tmask = tree != nullptr && trow < T ? tree[trow] : 0ull;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nk && ok; ++j) {
            if (!(ok = warp_wait(&sfull[t], uint32_t(j & 1)))) break;
            tc::tc_fence_after();
            float sv[AP_BN];
            ap_ld128(st, sv);
            if (tree != nullptr) {
                if (AP_BN * j + AP_BN - 1 >= start) {
#pragma unroll
                    for (int i = 0; i < AP_BN; ++i) {
                        const int kk = AP_BN * j + i - start;
                        if (kk >= 0 && (kk >= 64 || !((tmask >> kk) & 1ull))) sv[i] = -INFINITY;
                    }
                }
            } else if (AP_BN * j + AP_BN - 1 > qmin) {   // the tile crosses the diagonal: keys after the row's position
#pragma unroll
                for (int i = 0; i < AP_BN; ++i)
                    if (AP_BN * j + i > qpos) sv[i] = -INFINITY;
            }
            // eight independent max chains (the max has a fixed latency; one chain would serialize 64 of them)
            float mx[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) mx[c] = fmaxf(sv[2 * c], sv[2 * c + 1]);
#pragma unroll
            for (int c = 8; c < AP_BN / 2; ++c) mx[c & 7] = ap_max3(mx[c & 7], sv[2 * c], sv[2 * c + 1]);
            const float bm = fmaxf(ap_max3(mx[0], mx[1], mx[2]), ap_max3(mx[3], mx[4], ap_max3(mx[5], mx[6], mx[7])));
            const float m_new = fmaxf(m, bm * scale_log2);
            const bool need = m_new > m + AP_TAU;
            float factor = 1.f;
            if (need) {
                factor = ex2_approx(m - m_new);
                m = m_new;
                l *= factor;
            }
            if (j > 0 && __any_sync(0xffffffffu, need)) {   // O complete up to key tile j - 1, then rescaled
                if (!(ok = warp_wait(&pvdone[t], uint32_t((j - 1) & 1)))) break;
                tc::tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < AP_D / 32; ++c) {
                    uint32_t r[32];
                    tc::tmem_ld32(ot + uint32_t(c * 32), r);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
                    tc::tmem_st32(ot + uint32_t(c * 32), r);
                }
            }
            const float mneg = m == -INFINITY ? 0.f : -m;
            const uint64_t sl2 = ap_pack(scale_log2, scale_log2), nm2 = ap_pack(mneg, mneg);
            uint64_t ls[4] = {ap_pack(0.f, 0.f), ap_pack(0.f, 0.f), ap_pack(0.f, 0.f), ap_pack(0.f, 0.f)};
            // P (BF16 pairs) over the first 64 columns of S_t, in two halves: the next S_t is issued after this P.V
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t pr[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int cc = 32 * hh + c;
                    float x0, x1, p0, p1;
                    ap_unpack(ap_fma2(ap_pack(sv[2 * cc], sv[2 * cc + 1]), sl2, nm2), x0, x1);
                    if (EMU == AP_EXP_H2) {
                        ap_exp2_h2(x0, x1, p0, p1);
                    } else if ((cc & 7) < EMU) {
                        ap_exp2_poly(x0, x1, p0, p1);
                    } else {
                        p0 = ex2_approx(x0);
                        p1 = ex2_approx(x1);
                    }
                    ls[c & 3] = ap_add2(ls[c & 3], ap_pack(p0, p1));
                    const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
                    pr[c] = *reinterpret_cast<const uint32_t *>(&b);
                }
                tc::tmem_st32(st + uint32_t(32 * hh), pr);
            }
            {
                float a0, a1, b0, b1;
                ap_unpack(ap_add2(ap_add2(ls[0], ls[1]), ap_add2(ls[2], ls[3])), a0, a1);
                l += a0 + a1;
            }
            tc::tmem_st_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&pfull[t]);
        }
        int good = ok ? 1 : 0;
        if (ok && lane == 0) good = tc::mbar_wait(&pvdone[t], uint32_t((nk - 1) & 1));
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good && lane == 0) fail();
        tc::tc_fence_after();
        if (good && !abort_flag) {
            const int qrow = q0 + t * AP_BM + row;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16 *dst = out + int64_t(qrow) * out_ts + int64_t(h) * out_hs;
#pragma unroll 1
            for (int c = 0; c < AP_D / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(ot + uint32_t(c * 32), r);
                tc::tmem_ld_wait();
                if (qrow < T) {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        __nv_bfloat162 o[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            o[u] = __floats2bfloat162_rn(__uint_as_float(r[8 * v + 2 * u]) * inv,
                                                         __uint_as_float(r[8 * v + 2 * u + 1]) * inv);
                        reinterpret_cast<uint4 *>(dst + c * 32)[v] = *reinterpret_cast<uint4 *>(o);
                    }
                }
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

}  // namespace xt

using namespace xt;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 ap_encode_fn() {
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

// [rows, 128] BF16 rows (contiguous) as 128-row x 64-value boxes, 128-byte swizzled
bool ap_map_rows(CUtensorMap *map, const void *ptr, uint64_t rows) {
    auto fn = ap_encode_fn();
    if (!fn || reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    cuuint64_t dims[2] = {cuuint64_t(AP_D), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(AP_D) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(AP_BN)};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [T, Hq, 128] BF16 view (unit stride along the head dim, element strides ts, hs) as a 3-D map (d, head, token) whose
// box is 128 tokens x 64 values of one head
bool ap_map_q(CUtensorMap *map, const void *ptr, int T, int Hq, int64_t ts, int64_t hs) {
    auto fn = ap_encode_fn();
    if (!fn || ts <= 0 || hs <= 0 || ts % 8 || hs % 8 || reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    cuuint64_t dims[3] = {cuuint64_t(AP_D), cuuint64_t(Hq), cuuint64_t(T)};
    cuuint64_t strides[2] = {cuuint64_t(hs) * 2, cuuint64_t(ts) * 2};
    cuuint32_t box[3] = {64, 1, cuuint32_t(AP_BM)};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" {

// Causal GQA attention of T queries at positions start .. start + T - 1 over a BF16 KV cache, head dim 128.
// q: [T, Hq, 128] view (unit stride along d, element strides q_ts, q_hs; multiples of 8). k, v: the cache as
// [kv_rows, 128] contiguous rows; key `key` of kv head g is row kv_row0 + g * kv_hs + key (a [B, Hkv, max_len, 128]
// cache: kv_row0 = b * Hkv * max_len, kv_hs = max_len). out: [T, Hq, 128] view (strides out_ts, out_hs).
// Query t attends to keys 0 .. start + t; start + T <= kv_hs. With tree_mask ([T] 64-bit words, T <= 64: a draft tree
// whose node i sits in cache slot start + i), query t attends to keys 0 .. start - 1 and to slot start + i where bit i
// of tree_mask[t] is set (its ancestors and itself).
int xt_attn_prefill(const void *q, int64_t q_ts, int64_t q_hs, const void *k, const void *v, int64_t kv_rows,
                    int64_t kv_row0, int64_t kv_hs, int T, int start, int Hq, int Hkv, void *out, int64_t out_ts,
                    int64_t out_hs, float scale, const unsigned long long *tree_mask, int *error,
                    cudaStream_t stream) {
    if (T <= 0 || start < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || int64_t(start) + T > kv_hs) return -2;
    if (tree_mask && T > 64) return -2;
    if (kv_rows <= 0 || kv_rows > INT32_MAX || kv_row0 < 0 || kv_row0 + Hkv * kv_hs > kv_rows) return -2;
    if ((out_ts | out_hs) % 8 || reinterpret_cast<uintptr_t>(out) % 16) return -2;
    const int64_t nqt = (int64_t(T) + 2 * AP_BM - 1) / (2 * AP_BM);
    if (nqt * Hq > INT32_MAX) return -2;
    CUtensorMap mq, mk, mv;
    if (!ap_map_q(&mq, q, T, Hq, q_ts, q_hs) || !ap_map_rows(&mk, k, uint64_t(kv_rows)) ||
        !ap_map_rows(&mv, v, uint64_t(kv_rows)))
        return -3;
    // XTIER_ATTN_PREFILL_EMU (0-8): pairs of every 8 whose exponentials take the FMA-pipe polynomial; 9: every
    // exponential through the packed f16x2 MUFU operation (tuning)
    static const int emu = [] {
        const char *e = getenv("XTIER_ATTN_PREFILL_EMU");
        const int v = e && *e ? atoi(e) : AP_EMU;
        return v < 0 ? 0 : v > 9 ? 9 : v;
    }();
    auto launch = [&](auto kernel) {
        if (xt_smem_optin(kernel, int(ApSmem::BYTES)) != cudaSuccess) return -4;
        cudaFuncAttributes fa;   // the register split assumes exactly AP_REG_LAUNCH registers per thread at launch
        if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess || fa.numRegs != AP_REG_LAUNCH) return -5;
        kernel<<<unsigned(nqt * Hq), AP_THREADS, ApSmem::BYTES, stream>>>(
            mq, mk, mv, T, start, Hq, Hq / Hkv, int(kv_row0), int(kv_hs), scale * 1.4426950408889634f,
            static_cast<__nv_bfloat16 *>(out), out_ts, out_hs, tree_mask, error);
        return 0;
    };
    int rc;
    switch (emu) {
        case 0: rc = launch(attn_prefill_kernel<0>); break;
        case 1: rc = launch(attn_prefill_kernel<1>); break;
        case 2: rc = launch(attn_prefill_kernel<2>); break;
        case 3: rc = launch(attn_prefill_kernel<3>); break;
        case 4: rc = launch(attn_prefill_kernel<4>); break;
        case 8: rc = launch(attn_prefill_kernel<8>); break;
        default: rc = launch(attn_prefill_kernel<AP_EXP_H2>); break;
    }
    if (rc) return rc;
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
