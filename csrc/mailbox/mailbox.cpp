// CPU<->GPU mailbox, host side (layout: csrc/include/xt_mailbox.h).
//
// One mailbox = one slot in mapped pinned memory + its device state + a dispatcher thread pinned to one CPU. GPU kernels
// (csrc/cuda/moe_decode.cu) publish requests; the dispatcher runs the registered CPU engine plan of the request's layer
// and answers. No host callback and no stream memory operation is involved, so the kernels on both sides are plain
// kernel nodes of a CUDA graph, and every GPU wait is bounded by the kernel's own deadline.
//
// The dispatcher also keeps per-layer decayed route counts of every call (all routes, GPU-served ones included), which
// the adaptive hot-slot policy reads, and can append a binary route trace (XTIER_ROUTE_TRACE) for the planner.
// Reference parity: csrc/mailbox/mailbox.cpp:73-106 (slots), :516-710 (dispatcher, stats), :33-50 (route trace),
// :684-706 (watchdog: here the GPU-side deadline plus the host check of the error words), :518-520 (debug stall).
#include <cuda_runtime.h>
#include <pthread.h>
#include <sched.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <atomic>
#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../include/xt_engine.h"
#include "../include/xt_mailbox.h"

namespace {

thread_local std::string g_err;

double now_us() {
    return std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

struct TraceHead {   // one record per CPU call, followed by m*k int32 routes as routed
    double t_us, wall_us;
    int32_t layer, m, k, groups;
};

struct LayerStats {
    void *plan = nullptr;
    int experts = 0;
    std::vector<float> counts;   // decayed route counts per expert
    double calls = 0, cpu_us = 0, cpu_routes = 0, gpu_routes = 0;
};

struct Mailbox {
    int hidden = 0;
    char *host = nullptr;   // the slot (mapped pinned)
    char *devp = nullptr;   // device-visible address of `host`
    XtMailboxDev *dev = nullptr;
    XtMailbox view{};
    std::thread thread;
    std::atomic<bool> stop{false};
    std::mutex mu;   // guards layers / counts between the dispatcher and readers
    std::unordered_map<int, LayerStats> layers;
    float decay = 1.f;
    int stall_us = 0;
    FILE *trace = nullptr;
    uint32_t last = 0;
    double calls = 0, errors = 0, wall_us = 0;

    XtMailboxHeader *hdr() { return reinterpret_cast<XtMailboxHeader *>(host); }
    uint16_t *x() { return reinterpret_cast<uint16_t *>(host + sizeof(XtMailboxHeader)); }
    int32_t *ids() { return reinterpret_cast<int32_t *>(x() + size_t(XT_MB_MAX_TOKENS) * hidden); }
    float *w() { return reinterpret_cast<float *>(ids() + XT_MB_MAX_TOKENS * XT_MB_MAX_ROUTES); }
    int32_t *orig() { return reinterpret_cast<int32_t *>(w() + XT_MB_MAX_TOKENS * XT_MB_MAX_ROUTES); }
    float *y() {
        size_t off = reinterpret_cast<char *>(orig() + XT_MB_MAX_TOKENS * XT_MB_MAX_ROUTES) - host;
        off = (off + 255) & ~size_t(255);
        return reinterpret_cast<float *>(host + off);
    }

    void serve(uint32_t seq) {
        XtMailboxHeader *h = hdr();
        const int layer = h->layer, m = h->m, k = h->k;
        const double t0 = now_us();
        if (stall_us > 0) {
            timespec ts{stall_us / 1000000, (stall_us % 1000000) * 1000L};
            nanosleep(&ts, nullptr);
        }
        int groups = -1;
        {
            std::lock_guard<std::mutex> lk(mu);
            auto it = layers.find(layer);
            if (it == layers.end() || !it->second.plan || m < 1 || m > XT_MB_MAX_TOKENS || k < 1 ||
                k > XT_MB_MAX_ROUTES || h->hidden != hidden) {
                h->cpu_error = 1;
                memset(y(), 0, sizeof(float) * size_t(XT_MB_MAX_TOKENS) * hidden);
            } else {
                LayerStats &L = it->second;
                groups = xt_engine_forward_decode(L.plan, m, k, x(), ids(), w(), y());
                if (groups < 0) {
                    h->cpu_error = 1;
                    memset(y(), 0, sizeof(float) * size_t(m) * hidden);
                }
                const double dt = now_us() - t0;
                L.calls += 1;
                L.cpu_us += dt;
                for (auto &c : L.counts) c *= decay;
                const int32_t *o = orig();
                const int32_t *cid = ids();
                for (int i = 0; i < m * k; ++i) {
                    if (o[i] >= 0 && o[i] < L.experts) L.counts[o[i]] += 1.f;
                    if (o[i] >= 0) (cid[i] >= 0 ? L.cpu_routes : L.gpu_routes) += 1;
                }
            }
        }
        if (trace) {
            TraceHead th{t0, now_us() - t0, layer, m, k, groups};
            fwrite(&th, sizeof th, 1, trace);
            fwrite(orig(), sizeof(int32_t), size_t(m) * k, trace);
        }
        calls += 1;
        wall_us += now_us() - t0;
        std::atomic_thread_fence(std::memory_order_release);
        h->resp = seq;
    }

    void loop(int cpu) {
        if (cpu >= 0) {
            cpu_set_t set;
            CPU_ZERO(&set);
            CPU_SET(cpu, &set);
            pthread_setaffinity_np(pthread_self(), sizeof set, &set);
        }
        XtMailboxHeader *h = hdr();
        int idle = 0;
        while (!stop.load(std::memory_order_relaxed)) {
            uint32_t req = h->req;
            if (req != last) {
                std::atomic_thread_fence(std::memory_order_acquire);
                last = req;
                serve(req);
                idle = 0;
            } else if (++idle > 100000) {
                // long idle (no decode running): back off so an idle server does not burn a core at full speed
                timespec ts{0, 20000};
                nanosleep(&ts, nullptr);
            } else {
                __builtin_ia32_pause();
            }
        }
    }
};

}  // namespace

extern "C" {

void *xt_mailbox_create(int hidden, double timeout_s) {
    if (hidden <= 0 || hidden % 8) {
        g_err = "mailbox: hidden must be a positive multiple of 8";
        return nullptr;
    }
    auto *mb = new Mailbox();
    mb->hidden = hidden;
    size_t bytes = xt_mb_bytes(hidden);
    if (cudaHostAlloc(reinterpret_cast<void **>(&mb->host), bytes, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        g_err = "mailbox: cudaHostAlloc failed";
        delete mb;
        return nullptr;
    }
    memset(mb->host, 0, bytes);
    if (cudaHostGetDevicePointer(reinterpret_cast<void **>(&mb->devp), mb->host, 0) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&mb->dev), sizeof(XtMailboxDev)) != cudaSuccess ||
        cudaMemset(mb->dev, 0, sizeof(XtMailboxDev)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        g_err = "mailbox: device setup failed";
        cudaFreeHost(mb->host);
        delete mb;
        return nullptr;
    }
    auto dv = [&](void *hp) { return mb->devp + (static_cast<char *>(hp) - mb->host); };
    mb->view.hdr = reinterpret_cast<XtMailboxHeader *>(mb->devp);
    mb->view.x = reinterpret_cast<uint16_t *>(dv(mb->x()));
    mb->view.ids = reinterpret_cast<int32_t *>(dv(mb->ids()));
    mb->view.w = reinterpret_cast<float *>(dv(mb->w()));
    mb->view.orig = reinterpret_cast<int32_t *>(dv(mb->orig()));
    mb->view.y = reinterpret_cast<float *>(dv(mb->y()));
    mb->view.dev = mb->dev;
    mb->view.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
    const char *st = getenv("XTIER_DEBUG_STALL_US");
    mb->stall_us = st ? atoi(st) : 0;
    const char *tr = getenv("XTIER_ROUTE_TRACE");
    if (tr && *tr) mb->trace = fopen(tr, "ab");
    return mb;
}

// Kernel-side view (device-visible pointers), copied into *out (sizeof(XtMailbox) bytes).
int xt_mailbox_view(void *h, void *out) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    memcpy(out, &mb->view, sizeof(XtMailbox));
    return int(sizeof(XtMailbox));
}

int xt_mailbox_register(void *h, int layer, void *plan, int experts) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    std::lock_guard<std::mutex> lk(mb->mu);
    LayerStats &L = mb->layers[layer];
    L.plan = plan;
    L.experts = experts;
    L.counts.assign(experts, 0.f);
    return 0;
}

int xt_mailbox_start(void *h, int cpu, float decay) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb || mb->thread.joinable()) return -1;
    mb->decay = decay;
    mb->stop.store(false);
    mb->last = mb->hdr()->req;
    mb->thread = std::thread([mb, cpu] { mb->loop(cpu); });
    return 0;
}

int xt_mailbox_stop(void *h) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    mb->stop.store(true);
    if (mb->thread.joinable()) mb->thread.join();
    return 0;
}

// out[8]: calls, mean wall us per call, cpu errors flagged, gpu timeouts flagged, total wall us, last seq, 0, 0
int xt_mailbox_stats(void *h, double *out) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    out[0] = mb->calls;
    out[1] = mb->calls ? mb->wall_us / mb->calls : 0;
    out[2] = mb->hdr()->cpu_error;
    out[3] = mb->hdr()->gpu_error;
    out[4] = mb->wall_us;
    out[5] = mb->hdr()->resp;
    out[6] = out[7] = 0;
    return 0;
}

// Decayed route counts of `layer` into counts[experts]; stats[4]: calls, cpu us, cpu routes, gpu routes.
int xt_mailbox_layer_stats(void *h, int layer, float *counts, double *stats) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    std::lock_guard<std::mutex> lk(mb->mu);
    auto it = mb->layers.find(layer);
    if (it == mb->layers.end()) return -1;
    if (counts) memcpy(counts, it->second.counts.data(), sizeof(float) * it->second.counts.size());
    if (stats) {
        stats[0] = it->second.calls;
        stats[1] = it->second.cpu_us;
        stats[2] = it->second.cpu_routes;
        stats[3] = it->second.gpu_routes;
    }
    return int(it->second.counts.size());
}

// Clears the error words (host and device) after the caller handled them.
int xt_mailbox_clear_errors(void *h) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    mb->hdr()->gpu_error = 0;
    mb->hdr()->cpu_error = 0;
    return cudaMemset(&mb->dev->error, 0, sizeof(uint32_t)) == cudaSuccess ? 0 : -1;
}

// Host copies of the slot arrays (tests: a host thread that plays the CPU side without an engine).
int xt_mailbox_host_ptrs(void *h, void **out) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    out[0] = mb->hdr();
    out[1] = mb->x();
    out[2] = mb->ids();
    out[3] = mb->w();
    out[4] = mb->orig();
    out[5] = mb->y();
    return 0;
}

int xt_mailbox_destroy(void *h) {
    auto *mb = static_cast<Mailbox *>(h);
    if (!mb) return -1;
    xt_mailbox_stop(h);
    cudaDeviceSynchronize();
    if (mb->trace) fclose(mb->trace);
    cudaFree(mb->dev);
    cudaFreeHost(mb->host);
    delete mb;
    return 0;
}

const char *xt_mailbox_error(void) { return g_err.c_str(); }

}  // extern "C"
