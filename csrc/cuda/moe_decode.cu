// Decode-time MoE on the GPU hot-slot pool (W4A16: FP4 weights x BF16 activations, FP32 sums), with the CPU tier
// reached through the mailbox. Three kernels per MoE call, all CUDA-graph capturable:
//
//   moe_route   one CTA per token: router logits (BF16 GEMV), softmax or grouped-sigmoid top-k, renormalization and
//               routed scale; each route is split by the residency table (GPU slot, or the CPU); tokens with CPU
//               routes are written into the mailbox slot and the last CTA publishes the request.
//   moe_gate_up one CTA per (route, block of I rows): SwiGLU(g13[0] * x.Wg, g13[1] * x.Wu) of the route's slot, FP32.
//   moe_down    one CTA per (token, block of H rows): sum over the token's GPU routes, in route order, of
//               w * g2 * mid.Wd; then (bounded) wait for the CPU part, add it, write BF16. No atomics: every output
//               element has one writer and a fixed summation order, so the result is deterministic.
//
// The GEMVs are weight-bandwidth bound at decode sizes (1-16 tokens per expert), so they run on CUDA cores with the
// hardware E2M1 and E4M3 conversions of sm_100: each lane streams 16-byte weight chunks (ld.global.nc, no L1
// allocation), converts 8 codes per cvt pair to f16x2, and accumulates one 16- (NVFP4) or 32-element (MXFP4) block in
// f16x2 before scaling into FP32. `LPR` lanes share a row (LPR * CH * 16 bytes = row bytes), so the activation slice
// of a lane stays in registers for all its rows.
// Reference parity: xtier/cache/pool.py:80-110 (_pack: residency split), :170-250 (_gate_up, _down, _combine),
// :251-258 (_unpack: CPU part + GPU part); xtier/backend/kernels.py:25-57 (mailbox pack/unpack).
#include "../include/xt_mailbox.h"
#include "common.cuh"
#include "params.h"
#include "fp4_stream.cuh"

#include <stdio.h>

namespace xt {


constexpr int ROUTE_THREADS = 512;
constexpr int ROUTE_WARPS = ROUTE_THREADS / 32;
constexpr int ROUTE_CLUSTER = 8;   // CTAs per token (a portable cluster size)
constexpr int MAX_E = 512;

// One warp selects token t's routes from its logits (shared `logits`, `sel` of E floats, `chosen`, `chosen_w` of k):
// selection values (softmax, or sigmoid + correction bias with group pruning), top-k (ties: lower id), weights
// (renormalized, scaled). Lane j < k + n_shared gets route j: (expert or -1 for a shared expert, weight, slot).
XT_DEV void route_select(const RouteParams &p, int t, float *logits, float *sel, int *chosen, float *chosen_w, int lane,
                         const int32_t *table, const float *corr, int &e_out, float &w_out, int &slot_out) {
    const int kk = p.k + p.n_shared;
    // scores -> selection values
    if (p.mode == 0) {   // softmax over all experts
        float mx = -INFINITY;
        for (int e = lane; e < p.E; e += 32) mx = fmaxf(mx, logits[e]);
        mx = warp_max(mx);
        float s = 0.f;
        for (int e = lane; e < p.E; e += 32) s += __expf(logits[e] - mx);
        s = warp_sum(s);
        for (int e = lane; e < p.E; e += 32) {
            float v = __expf(logits[e] - mx) / s;
            logits[e] = v;
            sel[e] = v;
        }
    } else {   // sigmoid scores; selection adds the correction bias; groups by the sum of their top two
        for (int e = lane; e < p.E; e += 32) {
            float v = 1.f / (1.f + __expf(-logits[e]));
            logits[e] = v;
            sel[e] = v + (corr ? corr[e] : 0.f);
        }
        __syncwarp();
        if (p.n_group > 1) {
            const int gs = p.E / p.n_group;
            float gscore = -INFINITY;
            if (lane < p.n_group) {
                float a = -INFINITY, b = -INFINITY;
                for (int e = lane * gs; e < (lane + 1) * gs; ++e) {
                    float v = sel[e];
                    if (v > a) {
                        b = a;
                        a = v;
                    } else if (v > b) {
                        b = v;
                    }
                }
                gscore = a + b;
            }
            unsigned keep = 0;
            for (int r = 0; r < p.topk_group; ++r) {
                float v = (lane < p.n_group && !((keep >> lane) & 1)) ? gscore : -INFINITY;
                float bv = v;
                int bi = lane;
                for (int o = 16; o > 0; o >>= 1) {
                    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                keep |= 1u << bi;
            }
            __syncwarp();
            for (int e = lane; e < p.E; e += 32)
                if (!((keep >> (e / gs)) & 1)) sel[e] = -INFINITY;
        }
    }
    __syncwarp();
    // top-k by selection value (ties: lower expert id)
    for (int r = 0; r < p.k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < p.E; e += 32)
            if (sel[e] > bv) {
                bv = sel[e];
                bi = e;
            }
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            const bool ok = bi < p.E && bv > -INFINITY;   // fewer eligible experts than k: a zero-weight route
            chosen[r] = ok ? bi : 0;
            chosen_w[r] = ok ? logits[bi] : 0.f;
            if (ok) sel[bi] = -INFINITY;
        }
        __syncwarp();
    }
    if (lane == 0) {
        float s = 0.f;
        for (int r = 0; r < p.k; ++r) s += chosen_w[r];
        float f = (p.renorm && s > 0.f ? 1.f / s : 1.f) * p.scale;
        for (int r = 0; r < p.k; ++r) chosen_w[r] *= f;
    }
    __syncwarp();
    e_out = -1;
    w_out = 0.f;
    slot_out = -1;
    if (lane < p.k && p.active && !p.active[t]) return;   // flagged off: no routed expert anywhere
    if (lane < p.k) {
        e_out = chosen[lane];
        w_out = chosen_w[lane];
        slot_out = table ? table[e_out] : e_out;
    } else if (lane < kk) {
        w_out = 1.f;
        slot_out = p.shared_slots[lane - p.k];
    }
}

// Prefill selection: logits precomputed (the FP32 router GEMM); one warp per token, eight tokens per CTA.
constexpr int SEL_WARPS = 8;

__global__ void __launch_bounds__(SEL_WARPS * 32) route_select_kernel(RouteParams p) {
    __shared__ float logits[SEL_WARPS][MAX_E];
    __shared__ float sel[SEL_WARPS][MAX_E];
    __shared__ int chosen[SEL_WARPS][XT_MB_MAX_ROUTES];
    __shared__ float chosen_w[SEL_WARPS][XT_MB_MAX_ROUTES];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x * SEL_WARPS + warp;
    if (t >= p.m) return;
    for (int e = lane; e < p.E; e += 32)
        logits[warp][e] = p.logits_in[size_t(t) * p.E + e] + (p.bias ? p.bias[e] : 0.f);
    __syncwarp();
    int e, slot;
    float wv;
    route_select(p, t, logits[warp], sel[warp], chosen[warp], chosen_w[warp], lane, p.table, p.corr, e, wv, slot);
    const int kk = p.k + p.n_shared;
    if (lane < kk) {
        const size_t o = size_t(t) * kk + lane;
        p.ids[o] = e;
        p.w[o] = wv;
        p.slots[o] = slot;
    }
}

// PCIe staging claim of expert e by one route: the first route of the call to name e takes the next staging index (or
// marks e "no room" past stage_max) and records e in claim order; a route that finds e being claimed waits (bounded)
// for the index. Negative: the route stays on the CPU tier (also when the wait runs out: the CPU then computes this
// token's route, the staged copy serves the others).
XT_DEV int stage_claim(const RouteParams &p, int e) {
    int v = atomicCAS(&p.claim[e], -1, -2);
    if (v == -1) {
        const int s = atomicAdd(p.claim_count, 1);
        if (s < p.E) p.claim_list[s] = e;
        const int r = s < p.stage_max ? s : -3;
        __threadfence();
        atomicExch(&p.claim[e], r);
        return r;
    }
    for (int i = 0; v == -2 && i < (1 << 16); ++i) v = *reinterpret_cast<volatile int *>(&p.claim[e]);
    return v;
}

// Decode router, one cluster of ROUTE_CLUSTER CTAs per token (blockIdx.y): every warp of the cluster computes whole
// expert rows (16-byte loads, all of a row's loads in flight, FP32 sums) and stores the logit straight into the
// leader CTA's shared memory (st.shared::cluster); one cluster barrier (release / acquire) hands them over, and the
// leader's warp 0 selects (route_select) and writes the routes. The leader also prefetches the bias, correction bias
// and residency table into its shared memory and, with the mailbox, copies the token's activations into the mapped
// slot of the CPU tier while the rows stream; the last token's leader publishes the request with one system-scope
// fence. No global scratch, counters or memory fences between CTAs.
__global__ void __cluster_dims__(ROUTE_CLUSTER, 1, 1) __launch_bounds__(ROUTE_THREADS, 1)
    moe_route_kernel(RouteParams p, XtMailbox mb, int use_mb) {
    __shared__ float logits[MAX_E];
    __shared__ float sel[MAX_E];
    __shared__ float bias_s[MAX_E];
    __shared__ float corr_s[MAX_E];
    __shared__ int32_t table_s[MAX_E];
    __shared__ int chosen[XT_MB_MAX_ROUTES];
    __shared__ float chosen_w[XT_MB_MAX_ROUTES];
    __shared__ int any_cpu;
    const int t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = tc::cluster_rank();
    const int kk = p.k + p.n_shared;
    const int chunks = p.H / 8;
    const uint4 *xg = reinterpret_cast<const uint4 *>(p.x + size_t(t) * p.H);
    // every CTA of the cluster must have started before the leader's shared memory is written remotely: arrive now,
    // wait just before the first remote store (the row loads overlap the barrier)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
    const int gw = int(rank) * ROUTE_WARPS + warp;
    // this warp's first router row (weights: independent of the previous kernel) is in flight before the wait
    uint4 r0[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = i * 32 + lane;
        r0[i] = (gw < p.E && c < chunks) ? ldg_nc_v4(reinterpret_cast<const uint4 *>(p.wr + size_t(gw) * p.H) + c)
                                         : make_uint4(0, 0, 0, 0);
    }
    pdl_wait();
    pdl_trigger();
    if (rank == 0) {
        if (use_mb) {   // PCIe writes overlap the logits; published below by this CTA
            uint4 *mbx = reinterpret_cast<uint4 *>(mb.x + size_t(t) * p.H);
            for (int i = tid; i < chunks; i += ROUTE_THREADS) mbx[i] = xg[i];
        }
        for (int e = tid; e < p.E; e += ROUTE_THREADS) {
            bias_s[e] = p.bias ? p.bias[e] : 0.f;
            corr_s[e] = p.corr ? p.corr[e] : 0.f;
            table_s[e] = p.table ? p.table[e] : e;
        }
        if (tid == 0) any_cpu = 0;
    }
    bool waited = false;
    for (int e = gw; e < p.E; e += ROUTE_CLUSTER * ROUTE_WARPS) {
        const uint4 *we = reinterpret_cast<const uint4 *>(p.wr + size_t(e) * p.H);
        float acc = 0.f;
        for (int c0 = 0; c0 < chunks; c0 += 32 * 8) {
            uint4 r[8], xv[8];
            const bool pre = e == gw && c0 == 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = c0 + i * 32 + lane;
                r[i] = pre ? r0[i] : (c < chunks ? ldg_nc_v4(we + c) : make_uint4(0, 0, 0, 0));
                xv[i] = c < chunks ? xg[c] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const __nv_bfloat162 *x2 = reinterpret_cast<const __nv_bfloat162 *>(&xv[i]);
                const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&r[i]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 fx = __bfloat1622float2(x2[j]), fw = __bfloat1622float2(w2[j]);
                    acc = fmaf(fx.x, fw.x, fmaf(fx.y, fw.y, acc));
                }
            }
        }
        acc = warp_sum(acc);
        if (!waited) {
            asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
            waited = true;
        }
        if (lane == 0)
            asm volatile("st.shared::cluster.f32 [%0], %1;\n" ::"r"(tc::mapa(&logits[e], 0)), "f"(acc) : "memory");
    }
    if (!waited) asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
    tc::cluster_sync();   // every logit is in the leader's shared memory
    if (rank != 0) return;
    for (int e = tid; e < p.E; e += ROUTE_THREADS) logits[e] += bias_s[e];
    __syncthreads();

    if (warp == 0) {
        int e, slot;
        float wv;
        route_select(p, t, logits, sel, chosen, chosen_w, lane, p.table ? table_s : nullptr, p.corr ? corr_s : nullptr,
                     e, wv, slot);
        if (p.share_min > 0 && p.cold_index) {   // miss share: the first CPU route goes to the GPU (host memory)
            const unsigned cm = __ballot_sync(0xffffffffu, lane < p.k && slot < 0 && e >= 0);
            if (__popc(cm) >= p.share_min && lane == __ffs(cm) - 1) {
                const int ci = p.cold_index[e];
                if (ci >= 0) slot = p.host_base + ci;
            }
        }
        if (p.stage_max > 0 && lane < p.k && slot < 0 && e >= 0 && p.cold_index[e] >= 0) {
            const int s = stage_claim(p, e);   // PCIe staging: the GPU computes it from a staged copy
            if (s >= 0) slot = p.stage_slot0 + s;
        }
        if (lane < kk) {
            const size_t o = size_t(t) * kk + lane;
            p.ids[o] = e;
            p.w[o] = wv;
            p.slots[o] = slot;
            if (use_mb) {
                const size_t mo = size_t(t) * kk + lane;   // [m, kk] as the engine takes it
                mb.ids[mo] = (slot < 0) ? e : -1;
                mb.w[mo] = wv;
                mb.orig[mo] = e;
                if (slot < 0 && e >= 0) atomicOr(&any_cpu, 1);
            }
        }
    }
    if (!use_mb) return;
    __syncthreads();
    // count the token as done; the last token of the call publishes it with a single system fence (x and the route
    // arrays were written by this CTA before the barrier above)
    if (tid == 0) {
        if (any_cpu) atomicOr(&mb.dev->any, 1u);
        if (p.m > 1) __threadfence_system();   // other tokens' leaders: their slot rows before the count
        const unsigned prev = atomicAdd(&mb.dev->done, 1u);
        if (prev == unsigned(p.m) - 1) {
            __threadfence();
            const unsigned any = atomicExch(&mb.dev->any, 0u);
            mb.dev->done = 0;
            mb.dev->pending = any;
            if (any) {
                const unsigned seq = mb.dev->seq + 1;
                mb.dev->seq = seq;
                mb.hdr->layer = p.layer;
                mb.hdr->m = p.m;
                mb.hdr->k = kk;
                mb.hdr->hidden = p.H;
                __threadfence_system();
                st_release_sys(&mb.hdr->req, seq);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ FP4 GEMV core
struct ExpertPtrs {
    const uint8_t *w;    // packed rows, row stride in bytes = K / 2
    const uint8_t *s;    // block scales, row stride K / bs
    size_t slot_w, slot_s;   // bytes between slots
};

// dot of one 16-byte chunk (32 elements) with 16 f16x2 activations; fmt 0 NVFP4 (two E4M3 scales), 1 MXFP4 (one)
XT_DEV float chunk_dot(uint4 wv, const __half2 (&x)[16], const uint8_t *sp, int fmt) {
    __half2 h[4];
    __half2 a0 = __float2half2_rn(0.f), a1 = __float2half2_rn(0.f);
    e2m1x8_to_h2(wv.x, h);
#pragma unroll
    for (int i = 0; i < 4; ++i) a0 = __hfma2(h[i], x[i], a0);
    e2m1x8_to_h2(wv.y, h);
#pragma unroll
    for (int i = 0; i < 4; ++i) a0 = __hfma2(h[i], x[4 + i], a0);
    e2m1x8_to_h2(wv.z, h);
#pragma unroll
    for (int i = 0; i < 4; ++i) a1 = __hfma2(h[i], x[8 + i], a1);
    e2m1x8_to_h2(wv.w, h);
#pragma unroll
    for (int i = 0; i < 4; ++i) a1 = __hfma2(h[i], x[12 + i], a1);
    float2 f0 = __half22float2(a0), f1 = __half22float2(a1);
    if (fmt == 0) {
        float2 s = e4m3x2_to_f2(*reinterpret_cast<const uint16_t *>(sp));
        return (f0.x + f0.y) * s.x + (f1.x + f1.y) * s.y;
    }
    return (f0.x + f0.y + f1.x + f1.y) * ue8m0_to_f(*sp);
}

template <int LPR, int CH>
XT_DEV void load_x_bf16(const __nv_bfloat16 *x, int q, __half2 (&xr)[CH][16]) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + size_t(c * LPR + q) * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint4 u = src[v];
            const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) xr[c][v * 4 + i] = __float22half2_rn(__bfloat1622float2(b[i]));
        }
    }
}

template <int LPR, int CH>
XT_DEV void load_x_f16(const __half *x, int q, __half2 (&xr)[CH][16]) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + size_t(c * LPR + q) * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const uint4 u = src[v];
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) xr[c][v * 4 + i] = h[i];
        }
    }
}

template <int LPR, int CH>
XT_DEV void load_x_f32(const float *x, int q, __half2 (&xr)[CH][16]) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const float4 *src = reinterpret_cast<const float4 *>(x + size_t(c * LPR + q) * 32);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            float4 f = src[v];
            xr[c][v * 2] = __floats2half2_rn(f.x, f.y);
            xr[c][v * 2 + 1] = __floats2half2_rn(f.z, f.w);
        }
    }
}

// One row: K = LPR * CH * 32 elements, lane q of its group covers chunks c*LPR+q. Returns the group-reduced sum.
template <int LPR, int CH>
XT_DEV float row_dot(const uint8_t *wrow, const uint8_t *srow, int fmt, int q, const __half2 (&xr)[CH][16]) {
    uint4 wv[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) wv[c] = ldg_nc_v4(wrow + size_t(c * LPR + q) * 16);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int chunk = c * LPR + q;
        const uint8_t *sp = fmt == 0 ? srow + chunk * 2 : srow + chunk;
        acc += chunk_dot(wv[c], xr[c], sp, fmt);
    }
    return group_sum<LPR>(acc);
}


// 16-byte load through the coherent path (pinned host memory read over PCIe)
XT_DEV uint4 ld_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Dot of a row whose chunks are already in registers (see gate_up: every row's loads are issued first).
template <int LPR, int CH>
XT_DEV float row_dot_loaded(const uint4 (&wv)[CH], const uint8_t *srow, int fmt, int q, const __half2 (&xr)[CH][16]) {
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int chunk = c * LPR + q;
        const uint8_t *sp = fmt == 0 ? srow + chunk * 2 : srow + chunk;
        acc += chunk_dot(wv[c], xr[c], sp, fmt);
    }
    return group_sum<LPR>(acc);
}

constexpr int GU_WARPS = 8;
constexpr int GU_U = 2;   // gate/up row pairs per warp step: 2 * GU_U rows of loads in flight per lane

template <int LPR, int CH>
__global__ void __launch_bounds__(GU_WARPS * 32) moe_gate_up_kernel(GateUpParams p) {
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    const int slot = p.slots[r];
    if (slot < 0) return;
    const int t = r / p.kk;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int RPW = 32 / LPR;   // rows per warp step
    const int q = lane % LPR, sub = lane / LPR;
    __half2 xr[CH][16];
    load_x_bf16<LPR, CH>(p.x + size_t(t) * p.H, q, xr);
    const int bs = p.fmt == 0 ? 16 : 32;
    const size_t wrow = p.H / 2, srow = p.H / bs;
    const uint8_t *w13 = p.w13, *s13 = p.s13;
    const float *g13 = p.g13;
    int ls = slot;
    const bool hostw = p.host && slot >= p.host_base;   // a CPU-tier expert shared with the GPU (PCIe loads)
    if (hostw) {
        ls = slot - p.host_base;
        w13 = reinterpret_cast<const uint8_t *>(p.host[0]);
        s13 = reinterpret_cast<const uint8_t *>(p.host[1]);
        g13 = reinterpret_cast<const float *>(p.host[2]);
    } else if (p.peer) {   // the slot's owner: this GPU or a peer (NVLink loads)
        const int o = slot / p.spr;
        ls = slot - o * p.spr;
        w13 = reinterpret_cast<const uint8_t *>(p.peer[o * 6 + 0]);
        s13 = reinterpret_cast<const uint8_t *>(p.peer[o * 6 + 1]);
        g13 = reinterpret_cast<const float *>(p.peer[o * 6 + 2]);
    }
    const uint8_t *W = w13 + size_t(ls) * 2 * p.I * wrow;
    const uint8_t *S = s13 + size_t(ls) * 2 * p.I * srow;
    const float gg = g13[2 * ls], gu = g13[2 * ls + 1];
    const int rows_per_cta = GU_WARPS * RPW * GU_U;
    int jr[GU_U], jj[GU_U];
    uint4 wg[GU_U][CH], wu[GU_U][CH];
#pragma unroll
    for (int u = 0; u < GU_U; ++u) {
        jr[u] = blockIdx.y * rows_per_cta + (warp * GU_U + u) * RPW + sub;
        jj[u] = min(jr[u], p.I - 1);   // every lane takes part in the group shuffles; out-of-range rows store nothing
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const uint8_t *pg = W + jj[u] * wrow + size_t(c * LPR + q) * 16;
            const uint8_t *pu = W + (p.I + jj[u]) * wrow + size_t(c * LPR + q) * 16;
            wg[u][c] = hostw ? ld_v4(pg) : ldg_nc_v4(pg);
            wu[u][c] = hostw ? ld_v4(pu) : ldg_nc_v4(pu);
        }
    }
#pragma unroll
    for (int u = 0; u < GU_U; ++u) {
        float g = row_dot_loaded<LPR, CH>(wg[u], S + jj[u] * srow, p.fmt, q, xr) * gg;
        float v = row_dot_loaded<LPR, CH>(wu[u], S + (p.I + jj[u]) * srow, p.fmt, q, xr) * gu;
        if (q == 0 && jr[u] < p.I) {
            if (p.limit > 0.f) {
                g = fminf(g, p.limit);
                v = fmaxf(-p.limit, fminf(v, p.limit));
            }
            const float h = (p.alpha == 1.f && p.beta == 0.f) ? g / (1.f + __expf(-g)) * v
                                                                : g / (1.f + __expf(-p.alpha * g)) * (v + p.beta);
            p.mid[size_t(r) * p.I + jj[u]] = __float2half_rn(h);
        }
    }
}


// One warp per route of the token (kk <= 16 warps); a CTA owns RPW*U output rows. Each warp loads its route's FP32
// intermediate slice and all U*CH weight chunks of its rows before any arithmetic; the per-route partial sums meet in
// shared memory and are added in route order (deterministic), then the CPU part and the optional extra term.
template <int LPR, int CH, int U>
__global__ void __launch_bounds__(XT_MB_MAX_ROUTES * 32) moe_down_kernel(DownParams p, XtMailbox mb, int use_mb) {
    constexpr int RPW = 32 / LPR;
    constexpr int ROWS = RPW * U;
    static_assert(ROWS % 4 == 0, "the epilogue writes four rows per thread");
    __shared__ float part[XT_MB_MAX_ROUTES][ROWS];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, j = threadIdx.x >> 5;   // warp j = route j
    const int q = lane % LPR, sub = lane / LPR;
    const int bs = p.fmt == 0 ? 16 : 32;
    const size_t wrow = p.I / 2, srow = p.I / bs;
    const int hb = blockIdx.y * ROWS;
    const int r = t * p.kk + j;
    const int slot = p.slots[r];
    if (slot >= 0) {   // warp-uniform
        const uint8_t *w2 = p.w2, *s2 = p.s2;
        const float *g2 = p.g2;
        int ls = slot;
        const bool hostw = p.host && slot >= p.host_base;
        if (hostw) {
            ls = slot - p.host_base;
            w2 = reinterpret_cast<const uint8_t *>(p.host[3]);
            s2 = reinterpret_cast<const uint8_t *>(p.host[4]);
            g2 = reinterpret_cast<const float *>(p.host[5]);
        } else if (p.peer) {
            const int o = slot / p.spr;
            ls = slot - o * p.spr;
            w2 = reinterpret_cast<const uint8_t *>(p.peer[o * 6 + 3]);
            s2 = reinterpret_cast<const uint8_t *>(p.peer[o * 6 + 4]);
            g2 = reinterpret_cast<const float *>(p.peer[o * 6 + 5]);
        }
        const uint8_t *W = w2 + size_t(ls) * p.H * wrow;
        const uint8_t *S = s2 + size_t(ls) * p.H * srow;
        uint4 wv[U][CH];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int h = min(hb + u * RPW + sub, p.H - 1);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const uint8_t *pw = W + h * wrow + size_t(c * LPR + q) * 16;
                wv[u][c] = hostw ? ld_v4(pw) : ldg_nc_v4(pw);
            }
        }
        __half2 xr[CH][16];
        load_x_f16<LPR, CH>(p.mid + size_t(r) * p.I, q, xr);
        const float wt = p.w[r] * g2[ls];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int h = min(hb + u * RPW + sub, p.H - 1);
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int chunk = c * LPR + q;
                const uint8_t *sp = p.fmt == 0 ? S + h * srow + chunk * 2 : S + h * srow + chunk;
                acc += chunk_dot(wv[u][c], xr[c], sp, p.fmt);
            }
            acc = group_sum<LPR>(acc);
            if (q == 0) part[j][u * RPW + sub] = wt * acc;
        }
    } else if (lane < RPW) {
#pragma unroll
        for (int u = 0; u < U; ++u) part[j][u * RPW + lane] = 0.f;
    }
    __syncthreads();
    // with a CPU part pending, this kernel leaves the sum to moe_combine (one poller per token instead of every CTA
    // polling host memory); otherwise it writes the final rows itself
    const bool defer = use_mb && mb.dev->pending;
    for (int i = threadIdx.x; i * 4 < ROWS; i += blockDim.x) {
        const int h = hb + i * 4;
        if (h >= p.H) break;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int jj = 0; jj < p.kk; ++jj)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] += part[jj][i * 4 + e];
        const size_t o = size_t(t) * p.H + h;
        if (p.out_f32) *reinterpret_cast<float4 *>(p.out_f32 + o) = make_float4(v[0], v[1], v[2], v[3]);
        if (defer) {
            *reinterpret_cast<float4 *>(p.gpu_part + o) = make_float4(v[0], v[1], v[2], v[3]);
            continue;
        }
        if (p.add) {
            uint2 a = *reinterpret_cast<const uint2 *>(p.add + o);
            const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(&a);
            float2 f0 = __bfloat1622float2(a2[0]), f1 = __bfloat1622float2(a2[1]);
            v[0] += f0.x;
            v[1] += f0.y;
            v[2] += f1.x;
            v[3] += f1.y;
        }
        __nv_bfloat162 r0 = __floats2bfloat162_rn(v[0], v[1]), r1 = __floats2bfloat162_rn(v[2], v[3]);
        uint2 outv;
        outv.x = *reinterpret_cast<uint32_t *>(&r0);
        outv.y = *reinterpret_cast<uint32_t *>(&r1);
        *reinterpret_cast<uint2 *>(p.out + o) = outv;
    }
}

// out[t] = GPU part + CPU part (+ add), one CTA per token. Only when the call has a CPU part: thread 0 waits for the
// dispatcher's answer with a deadline (a timeout sets the error words and the CPU part is left out), then the CTA reads
// the token's FP32 CPU row from mapped host memory in 16-byte pieces.
__global__ void __launch_bounds__(256) moe_combine_kernel(const float *gpu_part, const __nv_bfloat16 *add,
                                                          __nv_bfloat16 *out, int H, XtMailbox mb) {
    pdl_wait();
    if (!mb.dev->pending) return;
    __shared__ int ok;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        int got = 0;
        const unsigned seq = mb.dev->seq;
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
            if (ld_acquire_sys(&mb.hdr->resp) == seq) {
                got = 1;
                break;
            }
            if (globaltimer_ns() - t0 > mb.timeout_ns) {
                atomicExch(&mb.dev->error, 1u);
                mb.hdr->gpu_error = 1;
                break;
            }
        }
        ok = got;
    }
    __syncthreads();
    for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
        const size_t o = size_t(t) * H + h;
        float4 v = *reinterpret_cast<const float4 *>(gpu_part + o);
        if (ok) {
            float4 c;
            asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];\n"
                         : "=f"(c.x), "=f"(c.y), "=f"(c.z), "=f"(c.w)
                         : "l"(mb.y + o));
            v.x += c.x;
            v.y += c.y;
            v.z += c.z;
            v.w += c.w;
        }
        if (add) {
            uint2 a = *reinterpret_cast<const uint2 *>(add + o);
            const __nv_bfloat162 *a2 = reinterpret_cast<const __nv_bfloat162 *>(&a);
            float2 f0 = __bfloat1622float2(a2[0]), f1 = __bfloat1622float2(a2[1]);
            v.x += f0.x;
            v.y += f0.y;
            v.z += f1.x;
            v.w += f1.y;
        }
        __nv_bfloat162 r0 = __floats2bfloat162_rn(v.x, v.y), r1 = __floats2bfloat162_rn(v.z, v.w);
        uint2 outv;
        outv.x = *reinterpret_cast<uint32_t *>(&r0);
        outv.y = *reinterpret_cast<uint32_t *>(&r1);
        *reinterpret_cast<uint2 *>(out + o) = outv;
    }
}

}  // namespace xt

// ------------------------------------------------------------------------------------------------ host launchers
using namespace xt;

static int pick_lpr(int row_bytes, int *ch) {
    const int chunks = row_bytes / 16;
    if (row_bytes % 16) return 0;
    for (int lpr : {32, 16, 8, 4}) {
        if (chunks % lpr == 0 && chunks / lpr <= 8) {
            *ch = chunks / lpr;
            return lpr;
        }
    }
    return 0;
}

#define XT_GU_CASE(L, C)                                                                        \
    if (lpr == L && ch == C) {                                                                  \
        constexpr int rows = GU_WARPS * (32 / L) * GU_U;                                        \
        dim3 grid(p.routes, (p.I + rows - 1) / rows);                                           \
        return xt_launch(moe_gate_up_kernel<L, C>, grid, dim3(GU_WARPS * 32), 0, stream, p) ==   \
                       cudaSuccess                                                              \
                   ? 0                                                                          \
                   : -1;                                                                        \
    }

#define XT_DN_CASE(L, C, U)                                                                     \
    if (lpr == L && ch == C) {                                                                  \
        constexpr int rows = (32 / L) * U;                                                      \
        dim3 grid(m, (p.H + rows - 1) / rows);                                                  \
        if (xt_launch(moe_down_kernel<L, C, U>, grid, dim3(32 * p.kk), 0, stream, p, mb, use_mb) !=  \
            cudaSuccess)                                                                        \
            return -1;                                                                          \
        if (use_mb && xt_launch(moe_combine_kernel, dim3(m), dim3(256), 0, stream, p.gpu_part,    \
                                static_cast<const __nv_bfloat16 *>(p.add), p.out, p.H, mb) !=   \
                          cudaSuccess)                                                          \
            return -1;                                                                          \
        return 0;                                                                               \
    }

extern "C" {

int xt_moe_route(const RouteParams *p, const XtMailbox *mb, int use_mb, cudaStream_t stream) {
    if (p->E > MAX_E || p->H % 256 || p->H > 8192 || p->k + p->n_shared > XT_MB_MAX_ROUTES || p->k > 32) return -2;
    if (use_mb && p->m > XT_MB_MAX_TOKENS) return -3;
    if (!p->ws_logits || !p->ws_count) return -5;
    XtMailbox empty{};
    if (p->logits_in) {
        if (use_mb) return -6;
        route_select_kernel<<<(p->m + SEL_WARPS - 1) / SEL_WARPS, SEL_WARPS * 32, 0, stream>>>(*p);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    if (xt_launch(moe_route_kernel, dim3(ROUTE_CLUSTER, p->m), dim3(ROUTE_THREADS), 0, stream, *p,
                  use_mb ? *mb : empty, use_mb) != cudaSuccess)
        return -1;
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int xt_moe_gate_up(const GateUpParams *pp, cudaStream_t stream) {
    GateUpParams p = *pp;
    int ch = 0;
    int lpr = pick_lpr(p.H / 2, &ch);
    if ((p.fmt == 0 && p.H % 16) || (p.fmt == 1 && p.H % 32)) return -2;
    XT_GU_CASE(32, 1) XT_GU_CASE(32, 2) XT_GU_CASE(32, 3) XT_GU_CASE(32, 4) XT_GU_CASE(32, 5) XT_GU_CASE(32, 6)
    XT_GU_CASE(32, 7) XT_GU_CASE(32, 8) XT_GU_CASE(16, 1) XT_GU_CASE(16, 3) XT_GU_CASE(16, 5) XT_GU_CASE(16, 7)
    XT_GU_CASE(8, 1) XT_GU_CASE(8, 3) XT_GU_CASE(8, 5) XT_GU_CASE(8, 7) XT_GU_CASE(4, 1) XT_GU_CASE(4, 3)
    XT_GU_CASE(4, 5) XT_GU_CASE(4, 7)
    return -4;
}

int xt_moe_down(const DownParams *pp, const XtMailbox *mbp, int use_mb, int m, cudaStream_t stream) {
    DownParams p = *pp;
    XtMailbox mb = use_mb ? *mbp : XtMailbox{};
    int ch = 0;
    int lpr = pick_lpr(p.I / 2, &ch);
    if (p.kk > XT_MB_MAX_ROUTES) return -2;
    if (use_mb && !p.gpu_part) return -5;
    XT_DN_CASE(32, 1, 8) XT_DN_CASE(32, 2, 8) XT_DN_CASE(32, 3, 4) XT_DN_CASE(32, 4, 4) XT_DN_CASE(32, 5, 4)
    XT_DN_CASE(32, 6, 4) XT_DN_CASE(32, 7, 4) XT_DN_CASE(32, 8, 4) XT_DN_CASE(16, 1, 8) XT_DN_CASE(16, 3, 4)
    XT_DN_CASE(16, 5, 2) XT_DN_CASE(16, 7, 2) XT_DN_CASE(8, 1, 8) XT_DN_CASE(8, 3, 2) XT_DN_CASE(8, 5, 2)
    XT_DN_CASE(8, 7, 2) XT_DN_CASE(4, 1, 4) XT_DN_CASE(4, 3, 2) XT_DN_CASE(4, 5, 2) XT_DN_CASE(4, 7, 1)
    return -4;
}

}  // extern "C"

// ================================================================================================ expert parallelism
// Four launches per MoE call on every rank (phase 0..3), all capturable in a CUDA graph:
//   0 ep_dispatch   routes of this rank's tokens -> stores of the token rows and route metadata straight into the
//                   owner ranks' receive slots (peer memory over NVLink), then a release flag per destination
//   1 ep_gate_up    persistent: waits (bounded) for every source's flag, then SwiGLU(gate, up) of every received route,
//                   weights streamed through a shared-memory ring by bulk copies (fp4_stream.cuh)
//   2 ep_down       persistent, same streaming: down projection of every received route; the epilogue stores the
//                   weighted FP32 rows into the source rank's return buffer, and the last CTA releases the flags
//   3 ep_combine    waits (bounded) for every owner's return flag, sums each token's routes in route order (+ add)
// The epoch in state[0] (advanced by the dispatch of every call, identically on every rank) tags the flags, so graph
// replays need no host involvement. Waits poll this rank's own memory (peers write into it), never a peer's.
namespace xt {

constexpr int EP_MAX_ROUTES = 1024;   // T * k per rank
constexpr int EP_MAX_W = 8;

XT_DEV uint8_t *ep_buf(const EpParams &p, int r) { return reinterpret_cast<uint8_t *>(p.peer[r]); }

XT_DEV bool ep_wait_flag(const volatile uint32_t *f, uint32_t epoch, unsigned long long timeout_ns) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f) != epoch) {
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
    return true;
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpParams p) {
    __shared__ int dest[EP_MAX_ROUTES], pos[EP_MAX_ROUTES];
    __shared__ bool last;
    const int n = p.T * p.k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int s = p.slots ? p.slots[i] : p.ids[i];
        dest[i] = s < 0 ? -1 : s / p.El;   // -1: the CPU tier computes this route (not dispatched)
    }
    __syncthreads();
    // slot of route i in its destination's region for this source (route order); only this CTA's routes
    for (int i = blockIdx.x * nw + (threadIdx.x >> 5); i < n; i += gridDim.x * nw) {
        int c = 0;
        for (int j = lane; j < i; j += 32) c += dest[j] == dest[i];
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0) pos[i] = c;
    }
    __syncthreads();
    for (int i = blockIdx.x * nw + warp; i < n; i += gridDim.x * nw) {
        const int d = dest[i], t = i / p.k;
        if (d < 0) continue;
        uint8_t *base = ep_buf(p, d);
        const size_t slot = size_t(p.rank) * p.R + pos[i];
        uint4 *dst = reinterpret_cast<uint4 *>(base + p.off_rx + slot * p.H * 2);
        const uint4 *src = reinterpret_cast<const uint4 *>(p.x + size_t(t) * p.H);
        for (int c = lane; c < p.H / 8; c += 32) {   // BF16 in, f16 on the wire (the expert kernels compute in f16x2)
            uint4 v = src[c];
            const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&v);
            uint4 o;
            __half2 *h = reinterpret_cast<__half2 *>(&o);
#pragma unroll
            for (int q = 0; q < 4; ++q) h[q] = __float22half2_rn(__bfloat1622float2(b[q]));
            dst[c] = o;
        }
        if (lane == 0) {
            int4 m = make_int4((p.slots ? p.slots[i] : p.ids[i]) % p.El, t, i % p.k, __float_as_int(p.w[i]));
            *reinterpret_cast<int4 *>(base + p.off_meta + slot * 16) = m;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned prev = atomicAdd(&p.state[1], 1u);
        last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x < p.W) {
        const int d = threadIdx.x;
        int c = 0;
        for (int i = 0; i < n; ++i) c += dest[i] == d;
        const uint32_t epoch = p.state[0] + 1;
        uint8_t *base = ep_buf(p, d);
        *reinterpret_cast<volatile int *>(base + p.off_cnt + size_t(p.rank) * 128) = c;
        __threadfence_system();
        st_release_sys(reinterpret_cast<volatile uint32_t *>(base + p.off_flag + size_t(p.rank) * 128), epoch);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        p.state[0] = p.state[0] + 1;
        p.state[1] = 0;
    }
}

// every CTA: wait for all sources of this epoch, then read their counts into shared memory (prefix offsets)
XT_DEV bool ep_gather_counts(const EpParams &p, uint32_t epoch, int *off /*[W+1]*/) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        uint8_t *me = ep_buf(p, p.rank);
        for (int s = 0; s < p.W && good; ++s)
            good = ep_wait_flag(reinterpret_cast<const volatile uint32_t *>(me + p.off_flag + size_t(s) * 128), epoch,
                                p.timeout_ns);
        if (!good) atomicExch(p.error, 1);
        off[0] = 0;
        for (int s = 0; s < p.W; ++s)
            off[s + 1] = off[s] + (good ? *reinterpret_cast<const volatile int *>(me + p.off_cnt + size_t(s) * 128) : 0);
        ok = good;
    }
    __syncthreads();
    return ok;
}

XT_DEV void ep_locate(const EpParams &p, const int *off, int r, int &s, int &slot) {
    s = 0;
    while (s + 1 < p.W && r >= off[s + 1]) ++s;
    slot = s * p.R + (r - off[s]);
}

// Item order of the expert streams. The received routes are ordered by pool slot (a counting sort of their meta words
// in every CTA's shared memory) and a slot's routes take turns block by block: items (group g, row block b, member m)
// in that order. A block of weights is then copied for every route of its expert one after another by the same CTA,
// so the copies after the first hit L2 and each expert's weights cross HBM about once per call, however many tokens
// chose it. More routes than EP_MAX_SORT, or pools wider than EP_MAX_POOL: arrival order.
constexpr int EP_MAX_SORT = 2048;
constexpr int EP_MAX_POOL = 256;

struct EpSort {
    int ord[EP_MAX_SORT];        // received index of the i-th route in slot order
    int gstart[EP_MAX_POOL];     // first sorted index of group g
    int gsize[EP_MAX_POOL];      // routes of group g
    int ng;                      // groups (0: arrival order)
};

XT_DEV void ep_sort(const EpParams &p, const int *off, EpSort &S) {
    __shared__ int cnt[EP_MAX_POOL];
    const int n = off[p.W];
    const bool on = p.by_expert && n <= EP_MAX_SORT && p.El <= EP_MAX_POOL && n > 0;
    const uint8_t *me = ep_buf(p, p.rank);
    if (on) {
        for (int e = threadIdx.x; e < p.El; e += blockDim.x) cnt[e] = 0;
        __syncthreads();
        for (int r = threadIdx.x; r < n; r += blockDim.x) {
            int s, slot;
            ep_locate(p, off, r, s, slot);
            atomicAdd(&cnt[reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16)->x], 1);
        }
        __syncthreads();
        if (threadIdx.x == 0) {   // groups: the non-empty slots; cnt becomes each slot's next free sorted index
            int acc = 0, g = 0;
            for (int e = 0; e < p.El; ++e) {
                const int c = cnt[e];
                if (c) {
                    S.gstart[g] = acc;
                    S.gsize[g] = c;
                    ++g;
                }
                cnt[e] = acc;
                acc += c;
            }
            S.ng = g;
        }
        __syncthreads();
        // placement in arrival order within a slot (every CTA must derive the same item order): warp 0 walks the
        // routes 32 at a time; lanes with the same slot rank themselves by lane, the lowest one advances the slot
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            const unsigned below = (1u << lane) - 1u;
            for (int base = 0; base < n; base += 32) {
                const int r = base + lane;
                int e = -1;
                if (r < n) {
                    int s, slot;
                    ep_locate(p, off, r, s, slot);
                    e = reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16)->x;
                }
                const unsigned same = __match_any_sync(0xffffffffu, e);
                if (r < n) S.ord[cnt[e] + __popc(same & below)] = r;
                __syncwarp();
                if (r < n && (same & below) == 0) cnt[e] += __popc(same);
                __syncwarp();
            }
        }
    } else if (threadIdx.x == 0) {
        S.ng = 0;
    }
    __syncthreads();
}

// item -> (received route, row block)
XT_DEV void ep_item(const EpSort &S, int it, int nrb, int &r, int &rb) {
    if (S.ng == 0) {
        r = it / nrb;
        rb = it % nrb;
        return;
    }
    int lo = 0, hi = S.ng - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (S.gstart[mid] * nrb <= it) lo = mid;
        else hi = mid - 1;
    }
    const int local = it - S.gstart[lo] * nrb, sz = S.gsize[lo];
    rb = local / sz;
    r = S.ord[S.gstart[lo] + local % sz];
}

// Phase 1, persistent: items = (received route, R/2 rows of gate and the same R/2 rows of up) streamed through the
// shared-memory ring of fp4_stream.cuh; row group rs owns gate rows [rs*RPW/2, (rs+1)*RPW/2) and the matching up rows,
// so SwiGLU is applied where the sums meet. Each CTA takes a contiguous range of items (few route changes, so the
// activation slice and the metadata load rarely). mid is f16 [W*R, I].
template <int RPW>
__global__ void __launch_bounds__(fs::THREADS, 1) ep_gate_up_stream(EpParams p, fs::Geo geo) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int off[EP_MAX_W + 1];
    __shared__ volatile int abort_flag;
    __shared__ EpSort S;
    const uint32_t epoch = p.state[0];
    if (!ep_gather_counts(p, epoch, off)) return;
    ep_sort(p, off, S);
    const fs::Ring ring = fs::ring_init(smem_raw, geo, &abort_flag, p.error);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = geo.R / 2;
    const int nrb = p.I / half;
    const int items = off[p.W] * nrb;
    const int it0 = int((long long)items * blockIdx.x / gridDim.x);
    const int it1 = int((long long)items * (blockIdx.x + 1) / gridDim.x);
    const uint8_t *me = ep_buf(p, p.rank);
    fs::Cursor cur_ring;
    if (warp == fs::CW) {
        uint32_t filled = 0;
        int cur = -1, e = 0;
        for (int it = it0; it < it1; ++it) {
            int r, rb;
            ep_item(S, it, nrb, r, rb);
            if (r != cur) {
                int s, slot;
                ep_locate(p, off, r, s, slot);
                e = reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16)->x;
                cur = r;
            }
            const bool st = p.stage_base > 0 && e >= p.stage_base;   // a staging slot (host copy brought over PCIe)
            const uint8_t *w13 = st ? p.st_w13 : p.w13, *s13 = st ? p.st_s13 : p.s13;
            const size_t g0 = size_t(st ? e - p.stage_base : e) * 2 * p.I + size_t(rb) * half, u0 = g0 + p.I;
            const fs::Run runs[2] = {{w13 + g0 * geo.wrow, s13 + g0 * geo.srow, half, 0},
                                     {w13 + u0 * geo.wrow, s13 + u0 * geo.srow, half, half}};
            if (!fs::produce(ring, geo, runs, 2, cur_ring, filled)) break;
        }
        fs::produce_drain(ring, geo, filled);
        return;
    }
    fs::Lane L = fs::lane_setup(geo);
    constexpr int H2 = RPW / 2, STRIDE = 32 / RPW;
    int rows[RPW];
#pragma unroll
    for (int i = 0; i < H2; ++i) {
        rows[i] = L.rs * H2 + i;
        rows[H2 + i] = half + L.rs * H2 + i;
    }
    int cur = -1, slot = 0;
    float gg = 0.f, gu = 0.f;
    for (int it = it0; it < it1; ++it) {
        int r, rb;
        ep_item(S, it, nrb, r, rb);
        if (r != cur) {
            int s;
            ep_locate(p, off, r, s, slot);
            fs::lane_load_x(L, reinterpret_cast<const __half *>(me + p.off_rx + size_t(slot) * p.H * 2));
            const int e = reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16)->x;
            const bool stg = p.stage_base > 0 && e >= p.stage_base;
            const float *g13 = stg ? p.st_g13 + 2 * (e - p.stage_base) : p.g13 + 2 * e;
            gg = g13[0];
            gu = g13[1];
            cur = r;
        }
        float v;
        const int st = fs::consume<RPW>(ring, geo, L, rows, v, cur_ring);
        if (!st) break;
        const float u = __shfl_xor_sync(0xffffffffu, v, 16);
        if (st == 1 && lane < 16 && lane % STRIDE == 0) {
            const float g = v * gg, uu = u * gu;
            p.mid[size_t(slot) * p.I + rb * half + L.rs * H2 + lane / STRIDE] =
                __float2half_rn(g / (1.f + __expf(-g)) * uu);
        }
    }
}

// Phase 2, persistent: items = (received route, R rows of the down projection); row group rs owns rows
// [rs*RPW, (rs+1)*RPW) and stores them with one coalesced store straight into the source rank's return buffer (peer
// memory over NVLink). Every thread fences its stores at system scope before the CTA counts itself done; the last CTA
// releases every source's return flag.
template <int RPW>
__global__ void __launch_bounds__(fs::THREADS, 1) ep_down_stream(EpParams p, fs::Geo geo) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int off[EP_MAX_W + 1];
    __shared__ volatile int abort_flag;
    __shared__ bool last;
    __shared__ EpSort S;
    const uint32_t epoch = p.state[0];
    if (!ep_gather_counts(p, epoch, off)) return;
    ep_sort(p, off, S);
    const fs::Ring ring = fs::ring_init(smem_raw, geo, &abort_flag, p.error);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nrb = p.H / geo.R;
    const int items = off[p.W] * nrb;
    const int it0 = int((long long)items * blockIdx.x / gridDim.x);
    const int it1 = int((long long)items * (blockIdx.x + 1) / gridDim.x);
    const uint8_t *me = ep_buf(p, p.rank);
    fs::Cursor cur_ring;
    if (warp == fs::CW) {
        uint32_t filled = 0;
        int cur = -1, e = 0;
        for (int it = it0; it < it1; ++it) {
            int r, hb;
            ep_item(S, it, nrb, r, hb);
            if (r != cur) {
                int s, slot;
                ep_locate(p, off, r, s, slot);
                e = reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16)->x;
                cur = r;
            }
            const bool st = p.stage_base > 0 && e >= p.stage_base;
            const size_t row0 = size_t(st ? e - p.stage_base : e) * p.H + size_t(hb) * geo.R;
            const fs::Run run = {(st ? p.st_w2 : p.w2) + row0 * geo.wrow, (st ? p.st_s2 : p.s2) + row0 * geo.srow,
                                 geo.R, 0};
            if (!fs::produce(ring, geo, &run, 1, cur_ring, filled)) break;
        }
        fs::produce_drain(ring, geo, filled);
    } else {
        constexpr int STRIDE = 32 / RPW;
        fs::Lane L = fs::lane_setup(geo);
        int rows[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) rows[i] = L.rs * RPW + i;
        int cur = -1;
        float wt = 0.f;
        float *dst_row = nullptr;
        for (int it = it0; it < it1; ++it) {
            int r, hb;
            ep_item(S, it, nrb, r, hb);
            if (r != cur) {
                int s, slot;
                ep_locate(p, off, r, s, slot);
                fs::lane_load_x(L, p.mid + size_t(slot) * p.I);
                const int4 m = *reinterpret_cast<const int4 *>(me + p.off_meta + size_t(slot) * 16);
                wt = __int_as_float(m.w) *
                     (p.stage_base > 0 && m.x >= p.stage_base ? p.st_g2[m.x - p.stage_base] : p.g2[m.x]);
                dst_row = reinterpret_cast<float *>(ep_buf(p, s) + p.off_ret) + (size_t(m.y) * p.k + m.z) * p.H;
                cur = r;
            }
            float v;
            const int st = fs::consume<RPW>(ring, geo, L, rows, v, cur_ring);
            if (!st) break;
            if (st == 1 && lane % STRIDE == 0) dst_row[hb * geo.R + L.rs * RPW + lane / STRIDE] = v * wt;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(&p.state[8], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x < p.W) {
        if (threadIdx.x == 0) p.state[8] = 0;
        __threadfence_system();
        st_release_sys(reinterpret_cast<volatile uint32_t *>(ep_buf(p, threadIdx.x) + p.off_rflag +
                                                             size_t(p.rank) * 128),
                       epoch);
    }
}

__global__ void __launch_bounds__(256) ep_combine_kernel(EpParams p) {
    __shared__ int ok, cpu_ok;
    __shared__ unsigned gpu_mask;
    const int t = blockIdx.x;
    const uint32_t epoch = p.state[0];
    if (threadIdx.x == 0) {
        int good = 1;
        const uint8_t *me = ep_buf(p, p.rank);
        for (int d = 0; d < p.W && good; ++d)
            good = ep_wait_flag(reinterpret_cast<const volatile uint32_t *>(me + p.off_rflag + size_t(d) * 128), epoch,
                                p.timeout_ns);
        if (!good) atomicExch(p.error, 1);
        ok = good;
        unsigned mask = 0;   // routes computed on a GPU (the others went to the CPU tier and have no return row)
        for (int j = 0; j < p.k; ++j)
            if (!p.slots || p.slots[size_t(t) * p.k + j] >= 0) mask |= 1u << j;
        gpu_mask = mask;
        // the CPU tier's rows of this call: a bounded wait for the dispatcher's answer (a timeout sets the error
        // words and leaves the CPU part out)
        int got = 0;
        if (p.use_mb && p.mb.dev->pending) {
            const unsigned seq = p.mb.dev->seq;
            const uint64_t t0 = globaltimer_ns();
            for (;;) {
                if (ld_acquire_sys(&p.mb.hdr->resp) == seq) {
                    got = 1;
                    break;
                }
                if (globaltimer_ns() - t0 > p.mb.timeout_ns) {
                    atomicExch(&p.mb.dev->error, 1u);
                    p.mb.hdr->gpu_error = 1;
                    break;
                }
            }
        }
        cpu_ok = got;
    }
    __syncthreads();
    const float *ret = reinterpret_cast<const float *>(ep_buf(p, p.rank) + p.off_ret);
    const unsigned mask = gpu_mask;
    const int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4;   // four consecutive outputs per thread
    if (h >= p.H) return;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok)
        for (int j = 0; j < p.k; ++j)
            if (mask >> j & 1) {
                const float4 r = __ldcv(reinterpret_cast<const float4 *>(ret + (size_t(t) * p.k + j) * p.H + h));
                v.x += r.x;
                v.y += r.y;
                v.z += r.z;
                v.w += r.w;
            }
    const size_t o = size_t(t) * p.H + h;
    if (cpu_ok) {
        float4 c;
        asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];\n"
                     : "=f"(c.x), "=f"(c.y), "=f"(c.z), "=f"(c.w)
                     : "l"(p.mb.y + o));
        v.x += c.x;
        v.y += c.y;
        v.z += c.z;
        v.w += c.w;
    }
    if (p.add) {
        const uint2 a = *reinterpret_cast<const uint2 *>(p.add + o);
        const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.x));
        const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.y));
        v.x += a0.x;
        v.y += a0.y;
        v.z += a1.x;
        v.w += a1.y;
    }
    const __nv_bfloat162 r0 = __floats2bfloat162_rn(v.x, v.y), r1 = __floats2bfloat162_rn(v.z, v.w);
    *reinterpret_cast<uint2 *>(p.out + o) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&r0), *reinterpret_cast<const uint32_t *>(&r1));
}

}  // namespace xt

extern "C" int xt_ep_moe(const EpParams *pp, int phase, cudaStream_t stream) {
    EpParams p = *pp;
    if (p.W > EP_MAX_W || p.T * p.k > EP_MAX_ROUTES || p.H % 256 || p.I % 16 || p.k > 32) return -2;
    if (p.use_mb && p.T > XT_MB_MAX_TOKENS) return -2;
    if (phase == 0) {
        const int n = p.T * p.k;
        const int grid = (n + 7) / 8;   // one warp per route
        ep_dispatch_kernel<<<grid, 256, 0, stream>>>(p);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    if (phase == 3) {
        ep_combine_kernel<<<dim3(p.T, (p.H / 4 + 255) / 256), 256, 0, stream>>>(p);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    {
        const void *fns[4] = {reinterpret_cast<const void *>(ep_gate_up_stream<4>),
                              reinterpret_cast<const void *>(ep_gate_up_stream<8>),
                              reinterpret_cast<const void *>(ep_down_stream<4>),
                              reinterpret_cast<const void *>(ep_down_stream<8>)};
        for (const void *f : fns)
            if (xt_smem_optin(f, int(fs::SMEM_BYTES)) != cudaSuccess) return -5;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    fs::Geo geo;
    if (phase == 1) {
        if (!fs::make_geo(p.H, p.fmt, 2, geo) || p.I % (geo.R / 2)) return -3;
        if (geo.rpw == 8)
            ep_gate_up_stream<8><<<sms, fs::THREADS, fs::SMEM_BYTES, stream>>>(p, geo);
        else
            ep_gate_up_stream<4><<<sms, fs::THREADS, fs::SMEM_BYTES, stream>>>(p, geo);
    } else {
        if (!fs::make_geo(p.I, p.fmt, 1, geo) || p.H % geo.R) return -3;
        if (geo.rpw == 8)
            ep_down_stream<8><<<sms, fs::THREADS, fs::SMEM_BYTES, stream>>>(p, geo);
        else
            ep_down_stream<4><<<sms, fs::THREADS, fs::SMEM_BYTES, stream>>>(p, geo);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
