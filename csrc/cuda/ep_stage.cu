// PCIe staging of CPU-tier experts for the expert-parallel decode (sm_100a).
//
// With part of a layer's experts in the CPU engine's host memory, the CPU tier and the PCIe link can work on the
// same call: the router (moe_route, PCIe staging claim) hands up to stage_max of the CPU-tier experts its tokens chose
// to the GPU, and this kernel copies those experts from the engine's own slots -- host memory registered with CUDA and
// mapped into the device's address space, read in place over PCIe -- into GPU staging slots in the pool layout. The
// EP expert streams then compute their routes like any pool slot while the CPU engine computes the rest. Nothing is
// duplicated in host memory: the engine's slots are the only host copy.
//
// Grid (chunks, stage_max): CTA (c, s) copies part c of every piece of staged expert s (of every NUMA node's shard)
// with 16-byte loads, four in flight per thread; the global scales come from a small device table. The last CTA to
// finish resets the claims (every expert the call's routes claimed, staged or not) and the count for the next call.
// No CTA waits on another: the reset uses an arrival counter.
#include <cuda_runtime.h>

#include "common.cuh"
#include "params.h"

namespace xt {

constexpr int STAGE_THREADS = 256;

XT_DEV uint4 ld_sys_v4(const void *p) {   // host memory over PCIe (the coherent path)
    uint4 r;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Destination of piece q of node n inside staged expert s (the pool layout: w13 [2I, H/2] gate rows then up rows,
// s13 [2I, H/bs], w2 [H, I/2], s2 [H, I/bs]).
XT_DEV uint8_t *stage_dst(const StageParams &p, int s, int q, int n) {
    const size_t I = p.I, H = p.H;
    const size_t w13b = 2 * I * (H / 2), s13b = 2 * I * (H / p.bs), w2b = H * (I / 2), s2b = H * (I / p.bs);
    const size_t pb = p.piece_bytes[q];
    switch (q) {
        case 0: return p.w13 + s * w13b + n * pb;
        case 1: return p.w13 + s * w13b + I * (H / 2) + n * pb;
        case 2: return p.s13 + s * s13b + n * pb;
        case 3: return p.s13 + s * s13b + I * (H / p.bs) + n * pb;
        case 4: return p.w2 + s * w2b + n * pb;
        default: return p.s2 + s * s2b + n * pb;
    }
}

__global__ void __launch_bounds__(STAGE_THREADS) ep_stage_kernel(StageParams p) {
    __shared__ bool last;
    const int c = blockIdx.x, s = blockIdx.y;
    const int count = min(*p.claim_count, p.E);
    const int n_staged = min(count, p.stage_max);
    if (s < n_staged) {
        const int e = p.claim_list[s];
        const int es = p.cold_index[e];
        for (int n = 0; n < p.nodes; ++n) {
            const uint8_t *slot = reinterpret_cast<const uint8_t *>(p.base[n]) + size_t(es) * p.stride;
            for (int q = 0; q < 6; ++q) {
                const size_t bytes = p.piece_bytes[q];
                const size_t part = (bytes / 16 + p.chunks - 1) / p.chunks * 16;
                const size_t b0 = min(bytes, size_t(c) * part), b1 = min(bytes, b0 + part);
                const uint4 *src = reinterpret_cast<const uint4 *>(slot + p.piece_off[q] + b0);
                uint4 *dst = reinterpret_cast<uint4 *>(stage_dst(p, s, q, n) + b0);
                const int n16 = int((b1 - b0) / 16);
                int i = threadIdx.x;
                for (; i + 3 * STAGE_THREADS < n16; i += 4 * STAGE_THREADS) {
                    const uint4 a0 = ld_sys_v4(src + i), a1 = ld_sys_v4(src + i + STAGE_THREADS);
                    const uint4 a2 = ld_sys_v4(src + i + 2 * STAGE_THREADS);
                    const uint4 a3 = ld_sys_v4(src + i + 3 * STAGE_THREADS);
                    dst[i] = a0;
                    dst[i + STAGE_THREADS] = a1;
                    dst[i + 2 * STAGE_THREADS] = a2;
                    dst[i + 3 * STAGE_THREADS] = a3;
                }
                for (; i < n16; i += STAGE_THREADS) dst[i] = ld_sys_v4(src + i);
            }
        }
        if (c == 0 && threadIdx.x == 0) {
            p.g13[2 * s] = p.src_g13[2 * es];
            p.g13[2 * s + 1] = p.src_g13[2 * es + 1];
            p.g2[s] = p.src_g2[es];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(p.done, 1u) == gridDim.x * gridDim.y - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = threadIdx.x; i < count; i += STAGE_THREADS) p.claim[p.claim_list[i]] = -1;
    __syncthreads();
    if (threadIdx.x == 0) {
        *p.claim_count = 0;
        *p.done = 0;
    }
}

}  // namespace xt

extern "C" int xt_ep_stage(const xt::StageParams *pp, cudaStream_t stream) {
    const xt::StageParams &p = *pp;
    if (p.nodes < 1 || p.nodes > 8 || p.stage_max < 1 || p.chunks < 1 || p.E < 1 || (p.bs != 16 && p.bs != 32))
        return -2;
    if (p.stride % 16) return -3;
    for (int q = 0; q < 6; ++q)
        if (p.piece_off[q] % 16 || p.piece_bytes[q] % 16) return -3;
    for (int n = 0; n < p.nodes; ++n)
        if (p.base[n] % 16) return -3;
    xt::ep_stage_kernel<<<dim3(p.chunks, p.stage_max), xt::STAGE_THREADS, 0, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
