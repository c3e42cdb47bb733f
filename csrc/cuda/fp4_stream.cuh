// Weight streaming for FP4 expert GEMVs at decode sizes (one token per route, W4A16): a producer warp keeps a ring of
// shared-memory stages filled with bulk copies (cp.async.bulk, completing on an mbarrier) of the next block of R
// consecutive expert rows -- codes and block scales, one contiguous copy each per run of rows, so every request moves
// tens of kilobytes (small bulk copies cap the streaming rate well below HBM bandwidth) -- and sixteen consumer warps
// turn each stage into FP32 row sums. The copies read only this GPU's own memory.
//
// Consumer layout: the K chunks of a row (32 elements = 16 bytes each) are split over KS warps (KS = 1, 2, 4 or 8,
// enough that a warp covers at most 32 chunks) and the CW / KS warp groups take RPW rows each (R = RPW * CW / KS).
// A lane owns one chunk position for all of its rows and every item of a route: its slice of the activation vector
// (f16, 64 bytes) is loaded once per route and stays in registers. Per stage a lane does RPW chunk dots; the warp
// reduces its RPW partial rows with a butterfly (lane k * 32 / RPW ends with row k), and with KS > 1 the KS warps of a
// row group meet in shared memory, where the last to arrive adds the partials in warp order (deterministic).
//
// Every wait is bounded: a wait that runs out raises the CTA's abort flag and the error word, the producer waits
// (bounded) for its copies in flight, and the kernel returns.
#pragma once
#include "tc_common.cuh"

namespace xt {
namespace fs {

constexpr int CW = 16;                      // consumer warps
constexpr int THREADS = (CW + 1) * 32;      // + one producer warp
constexpr int MAX_STAGES = 8;
constexpr int RING_BYTES = 192 * 1024;      // stages share this
constexpr int SMEM_BYTES = RING_BYTES + 2 * MAX_STAGES * 8 + MAX_STAGES * CW * 8 * 4 + MAX_STAGES * CW * 4 + 256;

struct Geo {
    int K, fmt, bs;
    int chunks;      // K / 32
    int KS, cpw;     // warps per row, chunks per warp
    int rpw, R;      // rows per warp and per stage
    int wrow, srow;  // bytes per row: codes, scales
    int stage_bytes, stages;
};

// run_div: rows of a stage come in runs of R / run_div consecutive rows (gate/up: 2 runs). False if the shape cannot
// be streamed (then the caller uses another kernel).
__host__ __device__ inline bool make_geo(int K, int fmt, int run_div, Geo &g) {
    g.K = K;
    g.fmt = fmt;
    g.bs = fmt == 0 ? 16 : 32;
    if (K <= 0 || K % 32) return false;
    g.chunks = K / 32;
    const int need = (g.chunks + 31) / 32;
    g.KS = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 0;
    if (!g.KS) return false;
    g.cpw = (g.chunks + g.KS - 1) / g.KS;
    g.rpw = K >= 4096 ? 8 : 4;
    g.R = g.rpw * (CW / g.KS);
    g.wrow = K / 2;
    g.srow = K / g.bs;
    const int rr = g.R / run_div;
    if ((rr * g.wrow) % 16 || (rr * g.srow) % 16) return false;
    g.stage_bytes = (g.R * (g.wrow + g.srow) + 127) / 128 * 128;
    g.stages = RING_BYTES / g.stage_bytes;
    if (g.stages > MAX_STAGES) g.stages = MAX_STAGES;
    return g.stages >= 2;
}

// One run of `n` consecutive rows: codes at w, scales at s; lands at stage row `row0`.
struct Run {
    const uint8_t *w, *s;
    int n, row0;
};

struct Ring {
    uint8_t *stage;     // stages * stage_bytes, 128-byte aligned
    uint64_t *full, *empty;
    float *red;         // [MAX_STAGES][CW][8] partial rows of the KS warps of a row group
    int *cnt;           // [MAX_STAGES][CW] arrivals per row group
    volatile int *abort_flag;
    int *error;
};

// position in the ring: stage index and phase parity
struct Cursor {
    int s = 0;
    uint32_t ph = 0;
    XT_DEV void next(int stages) {
        if (++s == stages) {
            s = 0;
            ph ^= 1;
        }
    }
};

XT_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

// Carves the ring out of dynamic shared memory and initializes the barriers (whole CTA; ends with __syncthreads).
XT_DEV Ring ring_init(uint8_t *smem_raw, const Geo &g, volatile int *abort_flag, int *error) {
    Ring r;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    r.stage = base;
    r.full = reinterpret_cast<uint64_t *>(base + RING_BYTES);
    r.empty = r.full + MAX_STAGES;
    r.red = reinterpret_cast<float *>(r.empty + MAX_STAGES);
    r.cnt = reinterpret_cast<int *>(r.red + MAX_STAGES * CW * 8);
    r.abort_flag = abort_flag;
    r.error = error;
    for (int i = threadIdx.x; i < MAX_STAGES * CW; i += blockDim.x) r.cnt[i] = 0;
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < g.stages; ++s) {
            tc::mbar_init(&r.full[s], 1);
            tc::mbar_init(&r.empty[s], CW);
        }
        tc::fence_barrier_init();
    }
    __syncthreads();
    return r;
}

XT_DEV void ring_fail(const Ring &r) {
    *r.abort_flag = 1;
    atomicExch(r.error, 1);
}

// Producer side (the whole producer warp): one stage from `nruns` (<= 32) runs. Returns false on abort.
XT_DEV bool produce(const Ring &r, const Geo &g, const Run *runs, int nruns, Cursor &c, uint32_t &filled) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    if (lane == 0) ok = tc::mbar_wait(&r.empty[c.s], c.ph ^ 1);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok || *r.abort_flag) {
        if (lane == 0 && !ok) ring_fail(r);
        return false;
    }
    uint8_t *sw = r.stage + size_t(c.s) * g.stage_bytes;
    uint8_t *ss = sw + g.R * g.wrow;
    if (lane == 0) {
        int rows = 0;
        for (int i = 0; i < nruns; ++i) rows += runs[i].n;
        tc::mbar_arrive_expect_tx(&r.full[c.s], uint32_t(rows) * uint32_t(g.wrow + g.srow));
    }
    __syncwarp();
    if (lane < nruns) {
        const Run u = runs[lane];
        bulk_g2s(sw + size_t(u.row0) * g.wrow, u.w, uint32_t(u.n) * g.wrow, &r.full[c.s]);
        bulk_g2s(ss + size_t(u.row0) * g.srow, u.s, uint32_t(u.n) * g.srow, &r.full[c.s]);
    }
    __syncwarp();
    c.next(g.stages);
    ++filled;
    return true;
}

// After the producer's last stage, or an abort: wait (bounded) until every stage it filled has landed, so no copy is
// in flight into the shared memory of a CTA that exits.
XT_DEV void produce_drain(const Ring &r, const Geo &g, uint32_t filled) {
    if ((threadIdx.x & 31) != 0) return;
    const uint32_t n = filled < uint32_t(g.stages) ? filled : uint32_t(g.stages);
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t c = filled - 1 - i;
        tc::mbar_wait(&r.full[c % g.stages], (c / g.stages) & 1, 1u << 20);
    }
}

// dot of one 16-byte chunk (32 E2M1 codes) with 16 f16x2 activations, scaled: NVFP4 two E4M3 scales, MXFP4 one UE8M0
XT_DEV float chunk_dot_s(uint4 wv, const __half2 (&x)[16], const uint8_t *sp, int fmt) {
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
    const float2 f0 = __half22float2(a0), f1 = __half22float2(a1);
    if (fmt == 0) {
        const float2 sc = e4m3x2_to_f2(*reinterpret_cast<const uint16_t *>(sp));
        return (f0.x + f0.y) * sc.x + (f1.x + f1.y) * sc.y;
    }
    return (f0.x + f0.y + f1.x + f1.y) * ue8m0_to_f(*sp);
}

// Butterfly sum of N per-lane partial rows over the warp: lane k * (32 / N) ends with the full sum of row k.
template <int N>
XT_DEV float reduce_rows(const float (&v)[N]) {
    const int lane = threadIdx.x & 31;
    float a[N];
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = v[i];
#pragma unroll
    for (int n = N / 2, o = 16; n >= 1; n >>= 1, o >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int i = 0; i < n; ++i) {
            const float keep = up ? a[n + i] : a[i], send = up ? a[i] : a[n + i];
            a[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float k = a[0];
#pragma unroll
    for (int o = 16 / N; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
    return k;
}

// Consumer warp state: its place in the stage layout and its activation slice.
struct Lane {
    int ks, rs;        // K split index, row group
    int chunk;         // chunk of K this lane owns (valid if on)
    bool on;
    __half2 xr[16];
};

XT_DEV Lane lane_setup(const Geo &g) {
    Lane l;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    l.ks = warp % g.KS;
    l.rs = warp / g.KS;
    l.chunk = l.ks * g.cpw + lane;
    l.on = lane < g.cpw && l.chunk < g.chunks;
    return l;
}

// the lane's 32 activations of chunk l.chunk from an f16 vector [K] (coherent loads: in EP a peer stored the vector)
XT_DEV void lane_load_x(Lane &l, const __half *x) {
    if (!l.on) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + size_t(l.chunk) * 32);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const uint4 u = src[v];
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) l.xr[v * 4 + q] = h[q];
    }
}

// One stage: the N stage rows rows[0..N-1] against the lane's activation slice. Returns 1 when this warp holds the
// complete row sums (lane k * 32 / N has row k in `out`), 2 when another warp of the row group does, 0 on abort.
template <int N>
XT_DEV int consume(const Ring &r, const Geo &g, const Lane &l, const int (&rows)[N], float &out, Cursor &c) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = c.s;
    const uint32_t ph = c.ph;
    c.next(g.stages);
    if (!tc::mbar_wait(&r.full[s], ph)) {
        if (lane == 0) ring_fail(r);
        return 0;
    }
    float acc[N];
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = 0.f;
    if (l.on) {
        const uint8_t *sw = r.stage + size_t(s) * g.stage_bytes;
        const uint8_t *ss = sw + g.R * g.wrow;
        uint4 wv[N];
#pragma unroll
        for (int i = 0; i < N; ++i)
            wv[i] = *reinterpret_cast<const uint4 *>(sw + rows[i] * g.wrow + l.chunk * 16);
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint8_t *sp = ss + rows[i] * g.srow + (g.fmt == 0 ? l.chunk * 2 : l.chunk);
            acc[i] = chunk_dot_s(wv[i], l.xr, sp, g.fmt);
        }
    }
    out = reduce_rows<N>(acc);
    if (g.KS == 1) {
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&r.empty[s]);
        return 1;
    }
    // the KS warps of a row group: partials to shared memory; the last to arrive adds them in warp order
    constexpr int STRIDE = 32 / N;
    float *red = r.red + (size_t(s) * CW) * 8;
    if ((lane % STRIDE) == 0) red[warp * 8 + lane / STRIDE] = out;
    __threadfence_block();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&r.cnt[s * CW + l.rs], 1) == g.KS - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
        __threadfence_block();
        if ((lane % STRIDE) == 0) {
            float t = 0.f;
            for (int k = 0; k < g.KS; ++k)
                t += *reinterpret_cast<volatile float *>(&red[(l.rs * g.KS + k) * 8 + lane / STRIDE]);
            out = t;
        }
        if (lane == 0) r.cnt[s * CW + l.rs] = 0;
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&r.empty[s]);
    return last ? 1 : 2;
}

}  // namespace fs
}  // namespace xt
