// Speculative decoding: truncation of a chain draft at its confidence, before the target model's verify forward.
//
// Request b drafted S tokens (tokens[b, 1..S]; tokens[b, 0] is the last accepted token) with draft probabilities
// q[b, j, :]. keep = the number of leading drafts whose own probability q[b, j, tokens[b, 1 + j]] is at least the
// threshold, at least 1; all S when the request samples greedily (top_k == 1). The verify forward then computes only
// what the kept chain needs: flags[b, j] = (j <= keep) for the S + 1 verify tokens (a flag-0 token skips its routed
// experts in the MoE router), and the q row of the first dropped draft is zeroed, so the chain verifier rejects that
// proposal and resamples from the residual (p - q)+ = p: the verify is exactly that of the shorter chain (lossless).
// One CTA per request; the q row is cleared with 16-byte stores.
// (Reference parity: xtier/packs/speculative/truncate.py:1-60 -- same rule, flags and zeroed q row.)
#include "common.cuh"

namespace xt {

__global__ void __launch_bounds__(256) spec_truncate_kernel(float *__restrict__ q, const int64_t *__restrict__ tokens,
                                                           const int32_t *__restrict__ topk,
                                                           int32_t *__restrict__ flags, float th, long long stride_b,
                                                           long long stride_s, int V, int S) {
    const int b = blockIdx.x;
    __shared__ int keep_s;
    if (threadIdx.x < 32) {
        int first = S;
        for (int j = threadIdx.x; j < S; j += 32) {
            const long long tok = tokens[size_t(b) * (S + 1) + 1 + j];
            const float qv = (tok >= 0 && tok < V) ? q[b * stride_b + j * stride_s + tok] : 0.f;
            if (qv < th) first = min(first, j);
        }
        for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
        if (threadIdx.x == 0) {
            int keep = max(first, 1);
            if (topk && topk[b] == 1) keep = S;
            keep_s = keep;
        }
    }
    __syncthreads();
    const int keep = keep_s;
    for (int j = threadIdx.x; j <= S; j += blockDim.x) flags[size_t(b) * (S + 1) + j] = j <= keep ? 1 : 0;
    if (keep < S) {
        float *row = q + b * stride_b + keep * stride_s;
        if ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && V % 4 == 0) {
            float4 *r4 = reinterpret_cast<float4 *>(row);
            for (int i = threadIdx.x; i < V / 4; i += blockDim.x) r4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (int i = threadIdx.x; i < V; i += blockDim.x) row[i] = 0.f;
        }
    }
}

}  // namespace xt

using namespace xt;

extern "C" int xt_spec_truncate(float *q, const int64_t *tokens, const int32_t *topk, int32_t *flags, float th,
                                long long stride_b, long long stride_s, int B, int S, int V, cudaStream_t stream) {
    if (B < 0 || S < 1 || V < 1) return -2;
    if (B == 0) return 0;
    spec_truncate_kernel<<<B, 256, 0, stream>>>(q, tokens, topk, flags, th, stride_b, stride_s, V, S);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
