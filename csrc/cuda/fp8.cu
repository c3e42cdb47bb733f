// FP8 (E4M3) weights and rows.
//
// * fp8_rows: rows of an FP8 table with E8M0 block scales -> BF16, out[r] = e4m3(row) * 2^(e - 127) rounded to BF16
//   once. With `ids` it gathers rows [ids - lo] of a device table and zeroes ids outside [lo, hi) (a table sharded by
//   row range); without, it decodes rows already gathered (the row-table lookup's device buffer) in place order. One
//   thread per 16 payload bytes; the block size is a multiple of 16, so one scale per thread.
//   (Reference parity: xtier/packs/deepseek_v4/engram_gather.py:18-32 -- FP8 row x 2^(e-127) -> BF16, out-of-range
//   ids give zeros.)
// * gemv_fp8: decode projection with FP8 weights, y[m, N] = x[m, K] . (W[N, K] * S[N, K/128])^T (+ BF16 residual),
//   m <= 16 (W8A16). Same streaming structure as the BF16 GEMV (activations in shared memory, two rows per warp,
//   eight 16-byte loads per lane and row in flight before any arithmetic); each 16-element chunk's dot product is
//   scaled by its 128-column block scale and summed in FP32 in a fixed order, so the result does not depend on the
//   launch (deterministic; no split-K atomics).
// * fp8_dequant: W[N, K] * S[N, K/128] -> BF16, for prefill, where the projection is compute-bound and runs on the
//   tcgen05 BF16 GEMM.
//   (Reference parity: xtier/packs/glm5_next/fp8_weights.py:42-105 -- per row x 128-column scales, W8A16 decode.)
#include "common.cuh"

namespace xt {

__global__ void __launch_bounds__(256) fp8_rows_kernel(const uint8_t *__restrict__ tab, const uint8_t *__restrict__ sc,
                                                      const int64_t *__restrict__ ids, long long lo, long long hi,
                                                      int n, int dim, int blk, __nv_bfloat16 *__restrict__ out) {
    const int chunks = dim / 16;
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    if (i >= (long long)n * chunks) return;
    const int r = int(i / chunks), c = int(i % chunks);
    long long row = r;
    bool owned = true;
    if (ids) {
        const long long id = ids[r];
        owned = id >= lo && id < hi;
        row = owned ? id - lo : 0;
    }
    uint4 o[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (owned) {
        const uint4 v = ldg_nc_v4(tab + row * dim + c * 16);
        const float s = ue8m0_to_f(sc[row * (dim / blk) + (c * 16) / blk]);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        __nv_bfloat162 *ob = reinterpret_cast<__nv_bfloat162 *>(o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 a = e4m3x2_to_f2(uint16_t(w[q] & 0xffff));
            const float2 b = e4m3x2_to_f2(uint16_t(w[q] >> 16));
            ob[2 * q] = __floats2bfloat162_rn(a.x * s, a.y * s);
            ob[2 * q + 1] = __floats2bfloat162_rn(b.x * s, b.y * s);
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + size_t(r) * dim + c * 16);
    dst[0] = o[0];
    dst[1] = o[1];
}

constexpr int G8_WARPS = 8;
constexpr int G8_ROWS = 2;    // rows per warp
constexpr int G8_SEG = 8;     // 16-byte chunks per lane per row per segment (K segment = 4096 elements)

// dot of 16 E4M3 weights with 16 BF16 activations (two uint4 of x), FP32
XT_DEV float dot16(const uint4 &w, const uint4 &x0, const uint4 &x1) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    const __nv_bfloat162 *xa = reinterpret_cast<const __nv_bfloat162 *>(&x0);
    const __nv_bfloat162 *xb = reinterpret_cast<const __nv_bfloat162 *>(&x1);
    float a = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 w0 = e4m3x2_to_f2(uint16_t(ww[q] & 0xffff)), w1 = e4m3x2_to_f2(uint16_t(ww[q] >> 16));
        const __nv_bfloat162 *xs = q < 2 ? xa + 2 * q : xb + 2 * (q - 2);
        const float2 f0 = __bfloat1622float2(xs[0]), f1 = __bfloat1622float2(xs[1]);
        a = fmaf(w0.x, f0.x, fmaf(w0.y, f0.y, fmaf(w1.x, f1.x, fmaf(w1.y, f1.y, a))));
    }
    return a;
}

template <int M>
__global__ void __launch_bounds__(G8_WARPS * 32) gemv_fp8_kernel(const __nv_bfloat16 *__restrict__ x,
                                                                const uint8_t *__restrict__ W,
                                                                const float *__restrict__ S,
                                                                const __nv_bfloat16 *__restrict__ add,
                                                                __nv_bfloat16 *__restrict__ y, int N, int K) {
    extern __shared__ uint4 xs[];   // [M][K/8] BF16
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kx = K / 8, kc = K / 16, ks = K / 128;
    for (int i = threadIdx.x; i < M * kx; i += blockDim.x) xs[i] = reinterpret_cast<const uint4 *>(x)[i];
    __syncthreads();
    const int row0 = (blockIdx.x * G8_WARPS + warp) * G8_ROWS;
    if (row0 >= N) return;
    float acc[G8_ROWS][M];
#pragma unroll
    for (int r = 0; r < G8_ROWS; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[r][t] = 0.f;
    for (int seg = 0; seg < kc; seg += 32 * G8_SEG) {
        uint4 w[G8_ROWS][G8_SEG];
        float s[G8_ROWS][G8_SEG];
#pragma unroll
        for (int r = 0; r < G8_ROWS; ++r) {
            const int row = min(row0 + r, N - 1);
            const uint4 *wr = reinterpret_cast<const uint4 *>(W + size_t(row) * K);
#pragma unroll
            for (int c = 0; c < G8_SEG; ++c) {
                const int ci = seg + c * 32 + lane;
                w[r][c] = ci < kc ? ldg_nc_v4(wr + ci) : make_uint4(0, 0, 0, 0);
                s[r][c] = ci < kc ? __ldg(S + size_t(row) * ks + ci / 8) : 0.f;
            }
        }
#pragma unroll
        for (int c = 0; c < G8_SEG; ++c) {
            const int ci = seg + c * 32 + lane;
            if (ci >= kc) break;
#pragma unroll
            for (int t = 0; t < M; ++t) {
                const uint4 x0 = xs[t * kx + 2 * ci], x1 = xs[t * kx + 2 * ci + 1];
#pragma unroll
                for (int r = 0; r < G8_ROWS; ++r) acc[r][t] = fmaf(dot16(w[r][c], x0, x1), s[r][c], acc[r][t]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < G8_ROWS; ++r)
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

__global__ void __launch_bounds__(256) fp8_dequant_kernel(const uint8_t *__restrict__ W, const float *__restrict__ S,
                                                         __nv_bfloat16 *__restrict__ out, int N, int K) {
    const int chunks = K / 16;
    const long long i = blockIdx.x * 256ll + threadIdx.x;
    if (i >= (long long)N * chunks) return;
    const int r = int(i / chunks), c = int(i % chunks);
    const uint4 v = ldg_nc_v4(W + size_t(r) * K + c * 16);
    const float s = S[size_t(r) * (K / 128) + c / 8];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint4 o[2];
    __nv_bfloat162 *ob = reinterpret_cast<__nv_bfloat162 *>(o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 a = e4m3x2_to_f2(uint16_t(w[q] & 0xffff));
        const float2 b = e4m3x2_to_f2(uint16_t(w[q] >> 16));
        ob[2 * q] = __floats2bfloat162_rn(a.x * s, a.y * s);
        ob[2 * q + 1] = __floats2bfloat162_rn(b.x * s, b.y * s);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + size_t(r) * K + c * 16);
    dst[0] = o[0];
    dst[1] = o[1];
}

}  // namespace xt

using namespace xt;

extern "C" int xt_fp8_rows(const void *tab, const void *sc, const int64_t *ids, long long lo, long long hi, int n,
                           int dim, int blk, void *out, cudaStream_t stream) {
    if (n < 0 || dim % 16 || blk < 16 || blk % 16 || dim % blk) return -2;
    if (n == 0) return 0;
    const long long th = (long long)n * (dim / 16);
    fp8_rows_kernel<<<unsigned((th + 255) / 256), 256, 0, stream>>>(
        static_cast<const uint8_t *>(tab), static_cast<const uint8_t *>(sc), ids, lo, hi, n, dim, blk,
        static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int xt_gemv_fp8(const void *x, const void *W, const float *S, const void *add, void *y, int m, int N, int K,
                           cudaStream_t stream) {
    if (K % 128 || m < 1 || m > 16) return -2;
    const size_t smem = size_t(m) * K * 2;
    if (smem > 200 * 1024) return -3;
    const int rows_per_cta = G8_WARPS * G8_ROWS;
    dim3 grid((N + rows_per_cta - 1) / rows_per_cta);
    auto X = static_cast<const __nv_bfloat16 *>(x);
    auto Wp = static_cast<const uint8_t *>(W);
    auto A = static_cast<const __nv_bfloat16 *>(add);
    auto Y = static_cast<__nv_bfloat16 *>(y);
#define XT_G8(MM)                                                                                             \
    case MM: {                                                                                               \
        xt_smem_optin(gemv_fp8_kernel<MM>, 200 * 1024);                                                      \
        gemv_fp8_kernel<MM><<<grid, G8_WARPS * 32, smem, stream>>>(X, Wp, S, A, Y, N, K);                    \
        break;                                                                                               \
    }
    switch (m) {
        XT_G8(1) XT_G8(2) XT_G8(3) XT_G8(4) XT_G8(5) XT_G8(6) XT_G8(7) XT_G8(8)
        XT_G8(9) XT_G8(10) XT_G8(11) XT_G8(12) XT_G8(13) XT_G8(14) XT_G8(15) XT_G8(16)
        default: return -2;
    }
#undef XT_G8
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int xt_fp8_dequant(const void *W, const float *S, void *out, int N, int K, cudaStream_t stream) {
    if (K % 128 || N < 0) return -2;
    if (N == 0) return 0;
    const long long th = (long long)N * (K / 16);
    fp8_dequant_kernel<<<unsigned((th + 255) / 256), 256, 0, stream>>>(static_cast<const uint8_t *>(W), S,
                                                                        static_cast<__nv_bfloat16 *>(out), N, K);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
