// Skinny BF16 GEMM for decode: y[m, N] = x[m, K] . W[N, K]^T (+ optional BF16 residual add), m <= 16.
//
// At decode sizes the projection is a weight stream: every weight byte is read once and used by m <= 16 tokens, so
// the kernel is built to keep HBM busy rather than the tensor cores: the tokens' activations sit in shared memory,
// each warp owns 2 rows, its lanes stride K in 16-byte chunks, and all of a row pair's chunks of one K segment are
// loaded (ld.global.nc, no L1 allocation) before any arithmetic, so every warp has 16 independent 16-byte loads in
// flight. FP32 accumulation, one warp reduction per row and token.
// (The reference leaves these projections to SGLang's GEMMs; this is the decode-path replacement.)
#include "common.cuh"

namespace xt {

constexpr int GV_WARPS = 8;
constexpr int GV_ROWS = 2;        // rows per warp
constexpr int GV_SEG = 8;         // 16-byte chunks per lane per row per segment (K segment = 2048 elements)
constexpr int GV_MAX_WARPS = 16;  // a CTA whose activations fill most of an SM's shared memory runs 16 warps

template <int M, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) gemv_bf16_kernel(const __nv_bfloat16 *__restrict__ x,
                                                                 const __nv_bfloat16 *__restrict__ W,
                                                                 const __nv_bfloat16 *__restrict__ add,
                                                                 __nv_bfloat16 *__restrict__ y, int N, int K) {
    extern __shared__ uint4 xs[];   // [M][K/8]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kc = K / 8;
    const int row0 = (blockIdx.x * WARPS + warp) * GV_ROWS;
    // the first K segment's weights are in flight before the wait for the previous kernel (they do not depend on it)
    uint4 w[GV_ROWS][GV_SEG];
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r) {
        const int row = min(row0 + r, N - 1);
        const uint4 *wr = reinterpret_cast<const uint4 *>(W + size_t(row) * K);
#pragma unroll
        for (int c = 0; c < GV_SEG; ++c) {
            const int ci = c * 32 + lane;
            w[r][c] = (row0 < N && ci < kc) ? ldg_nc_v4(wr + ci) : make_uint4(0, 0, 0, 0);
        }
    }
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < M * kc; i += blockDim.x) xs[i] = reinterpret_cast<const uint4 *>(x)[i];
    __syncthreads();
    if (row0 >= N) return;
    float acc[GV_ROWS][M];
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[r][t] = 0.f;
    for (int seg = 0; seg < kc; seg += 32 * GV_SEG) {
        if (seg > 0) {
#pragma unroll
            for (int r = 0; r < GV_ROWS; ++r) {
                const int row = min(row0 + r, N - 1);
                const uint4 *wr = reinterpret_cast<const uint4 *>(W + size_t(row) * K);
#pragma unroll
                for (int c = 0; c < GV_SEG; ++c) {
                    const int ci = seg + c * 32 + lane;
                    w[r][c] = ci < kc ? ldg_nc_v4(wr + ci) : make_uint4(0, 0, 0, 0);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < GV_SEG; ++c) {
            const int ci = seg + c * 32 + lane;
            if (ci >= kc) break;
#pragma unroll
            for (int t = 0; t < M; ++t) {
                const uint4 xv = xs[t * kc + ci];
                const __nv_bfloat162 *x2 = reinterpret_cast<const __nv_bfloat162 *>(&xv);
#pragma unroll
                for (int r = 0; r < GV_ROWS; ++r) {
                    const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&w[r][c]);
                    float a = acc[r][t];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float2 fx = __bfloat1622float2(x2[i]), fw = __bfloat1622float2(w2[i]);
                        a = fmaf(fx.x, fw.x, fmaf(fx.y, fw.y, a));
                    }
                    acc[r][t] = a;
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) {
            float v = warp_sum(acc[r][t]);
            const int row = row0 + r;
            if (lane == t % 32 && row < N) {
                if (add) v += __bfloat162float(add[size_t(t) * N + row]);
                y[size_t(t) * N + row] = __float2bfloat16(v);
            }
        }
}

}  // namespace xt

using namespace xt;

extern "C" int xt_gemv_bf16(const void *x, const void *W, const void *add, void *y, int m, int N, int K,
                            cudaStream_t stream) {
    if (K % 8 || m < 1 || m > 16) return -2;
    const size_t smem = size_t(m) * K * 2;
    if (smem > 200 * 1024) return -3;
    // activations over 64 KB leave room for one or two CTAs per SM: those run 16 warps (up to 8 tokens, whose
    // registers fit 512 threads), so as many weight loads stay in flight as several 8-warp CTAs would keep
    const int warps = smem > 64 * 1024 && m <= 8 ? GV_MAX_WARPS : GV_WARPS;
    const int rows_per_cta = warps * GV_ROWS;
    dim3 grid((N + rows_per_cta - 1) / rows_per_cta);
    auto X = static_cast<const __nv_bfloat16 *>(x);
    auto Wp = static_cast<const __nv_bfloat16 *>(W);
    auto A = static_cast<const __nv_bfloat16 *>(add);
    auto Y = static_cast<__nv_bfloat16 *>(y);
#define XT_GV_LAUNCH(MM, WW)                                                                                  \
    {                                                                                                        \
        xt_smem_optin(gemv_bf16_kernel<MM, WW>, 200 * 1024);                                                 \
        if (xt_launch(gemv_bf16_kernel<MM, WW>, grid, dim3(WW * 32), smem, stream, X, Wp, A, Y, N, K) !=       \
            cudaSuccess)                                                                                     \
            return -1;                                                                                       \
    }
#define XT_GV(MM)                                                                                             \
    case MM:                                                                                                 \
        if (warps == GV_MAX_WARPS) XT_GV_LAUNCH(MM, GV_MAX_WARPS) else XT_GV_LAUNCH(MM, GV_WARPS)            \
        break;
#define XT_GV8(MM)                                                                                            \
    case MM:                                                                                                 \
        XT_GV_LAUNCH(MM, GV_WARPS)                                                                           \
        break;
    switch (m) {
        XT_GV(1) XT_GV(2) XT_GV(3) XT_GV(4) XT_GV(5) XT_GV(6) XT_GV(7) XT_GV(8)
        XT_GV8(9) XT_GV8(10) XT_GV8(11) XT_GV8(12) XT_GV8(13) XT_GV8(14) XT_GV8(15) XT_GV8(16)
        default: return -2;
    }
#undef XT_GV
#undef XT_GV8
#undef XT_GV_LAUNCH
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
