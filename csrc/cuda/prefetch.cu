// L2 prefetch of weights that a later kernel of the same CUDA graph will stream (sm_100a bulk prefetch).
//
// A decode step is a chain of short kernels whose cost is mostly the latency of the first weight bytes reaching the
// SMs. The next layer's dense weights (QKV and output projections, router) do not depend on anything computed in the
// current layer, so a side branch of the graph can pull them into L2 (126 MB on B200) while the current layer waits on
// something else -- in the tiered MoE, on the CPU experts. `cp.async.bulk.prefetch.L2.global` moves a contiguous
// range with one instruction and never blocks the issuing thread.
// (The reference uses the same instruction in its hyper-connection mix kernel, xtier/packs/qwen4_exp/hc_mix.py:27.)
#include "common.cuh"

namespace xt {

constexpr int PF_CHUNK = 32 * 1024;   // bytes per prefetch instruction

// regions: ptrs[i], bytes[i] (device arrays); the grid strides over all 32 KB chunks of all regions
__global__ void __launch_bounds__(128) l2_prefetch_kernel(const uint64_t *ptrs, const uint64_t *bytes, int n) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
    int chunk0 = 0;
    for (int r = 0; r < n; ++r) {
        const uint64_t base = ptrs[r], len = bytes[r];
        const int chunks = int((len + PF_CHUNK - 1) / PF_CHUNK);
        // this region's chunks that fall to this thread (global chunk index = chunk0 + c)
        int c = ((tid - chunk0) % nt + nt) % nt;
        for (; c < chunks; c += nt) {
            const uint64_t a = base + uint64_t(c) * PF_CHUNK;
            const uint64_t left = len - uint64_t(c) * PF_CHUNK;
            const uint32_t sz = uint32_t(left < PF_CHUNK ? left : PF_CHUNK) & ~15u;
            if (sz && (a & 15) == 0)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(sz) : "memory");
        }
        chunk0 = (chunk0 + chunks) % nt;
    }
}

}  // namespace xt

extern "C" int xt_l2_prefetch(const uint64_t *ptrs, const uint64_t *bytes, int n, int ctas, cudaStream_t stream) {
    if (n <= 0) return 0;
    xt::l2_prefetch_kernel<<<ctas > 0 ? ctas : 8, 128, 0, stream>>>(ptrs, bytes, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
