// Hot-slot swap ring: residency changes of the GPU expert pool applied by the GPU itself, so that the weight copies of
// a swap never sit on the decode stream.
//
// The host posts commands into a ring of mapped pinned memory (seq, layer, expert, slot; slot -1 unmaps) and bumps
// `posted`. pool_commit (one thread, graph capturable; the decode step runs it first) applies, in sequence order,
// every posted command whose copy has landed: an UNMAP at once, a MAP only once the side copy stream has written
// `landed` >= its sequence number (pool_landed, launched on that stream after the slot's copies). It writes the
// residency tables of the layers (`tables`: one device pointer per layer) and records how far it got in `applied`
// (device) and in a mapped word the host can read. A swap is: post UNMAP(victim) and apply it at once (a commit on the
// compute stream), make the copy stream wait for that, copy the incoming expert into the freed slot, pool_landed(seq
// of the MAP), post MAP(incoming, slot). Between the two, both experts route to the CPU tier; the slot is referenced by
// no table while it is rewritten. Reference parity: csrc/mailbox/mailbox.cpp:144-360 (posted / applied / landed
// sequence words of the pool command ring), xtier/cache/pool.py:112-142.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace xt {

struct RingState {
    int64_t applied;    // device: last sequence number applied
    int64_t landed;     // device: last MAP sequence number whose copies have landed
};

__global__ void pool_commit_kernel(const volatile int32_t *ring, const volatile int64_t *posted, int capacity,
                                   RingState *state, int32_t *const *tables, int n_tables,
                                   volatile int64_t *applied_host, int *error) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    pdl_wait();
    // In sequence order: every UNMAP at once (its own copy is about to overwrite the slot, even behind a MAP still in
    // flight), every MAP up to the first whose copy has not landed (copies land in sequence order, so the later MAPs
    // have not either). `applied` advances over the prefix applied in full; UNMAPs past it are applied again on the
    // next pass, in the same order relative to the MAPs, which leaves the tables as in-order application would.
    int64_t done = state->applied;
    bool blocked = false;
    const int64_t last = *posted;
    const int64_t landed = *reinterpret_cast<volatile int64_t *>(&state->landed);
    for (int64_t seq = done + 1; seq <= last; ++seq) {
        const volatile int32_t *e = ring + (seq % capacity) * 4;
        if (int64_t(uint32_t(e[0])) != (seq & 0xFFFFFFFFll)) break;   // the host has not finished writing it
        const int layer = e[1], expert = e[2], slot = e[3];
        if (slot >= 0 && (blocked || seq > landed)) {
            blocked = true;
            continue;
        }
        if (layer < 0 || layer >= n_tables || expert < 0) atomicExch(error, 3);
        else tables[layer][expert] = slot;
        if (!blocked) done = seq;
    }
    state->applied = done;
    __threadfence_system();
    *applied_host = done;
}

__global__ void pool_landed_kernel(RingState *state, int64_t seq) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        __threadfence();
        *reinterpret_cast<volatile int64_t *>(&state->landed) = seq;
    }
}

}  // namespace xt

using namespace xt;

extern "C" {

struct XtPoolRing {
    int32_t *ring_host = nullptr, *ring_dev = nullptr;   // [capacity][4] mapped
    int64_t *words_host = nullptr, *words_dev = nullptr; // mapped: [0] posted, [1] applied (GPU -> host)
    RingState *state = nullptr;                          // device
    int capacity = 0;
};

// A ring of `capacity` commands in mapped pinned memory plus its device state on the current device.
void *xt_pool_ring_create(int capacity) {
    if (capacity < 16) return nullptr;
    auto *r = new XtPoolRing();
    r->capacity = capacity;
    const size_t rb = size_t(capacity) * 4 * sizeof(int32_t);
    const unsigned flags = cudaHostAllocMapped | cudaHostAllocPortable;
    bool ok = cudaHostAlloc(reinterpret_cast<void **>(&r->ring_host), rb, flags) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void **>(&r->words_host), 2 * sizeof(int64_t), flags) == cudaSuccess;
    ok = ok && cudaHostGetDevicePointer(reinterpret_cast<void **>(&r->ring_dev), r->ring_host, 0) == cudaSuccess &&
         cudaHostGetDevicePointer(reinterpret_cast<void **>(&r->words_dev), r->words_host, 0) == cudaSuccess &&
         cudaMalloc(reinterpret_cast<void **>(&r->state), sizeof(RingState)) == cudaSuccess &&
         cudaMemset(r->state, 0, sizeof(RingState)) == cudaSuccess;
    if (!ok) {
        if (r->ring_host) cudaFreeHost(r->ring_host);
        if (r->words_host) cudaFreeHost(r->words_host);
        if (r->state) cudaFree(r->state);
        delete r;
        return nullptr;
    }
    for (int i = 0; i < capacity * 4; ++i) r->ring_host[i] = -1;
    r->words_host[0] = 0;
    r->words_host[1] = 0;
    return r;
}

void xt_pool_ring_destroy(void *h) {
    auto *r = static_cast<XtPoolRing *>(h);
    if (!r) return;
    cudaFreeHost(r->ring_host);
    cudaFreeHost(r->words_host);
    cudaFree(r->state);
    delete r;
}

// Host side: write command `seq` (1, 2, ...) and publish it. The caller keeps at most capacity - 1 commands unapplied.
int xt_pool_ring_post(void *h, int64_t seq, int layer, int expert, int slot) {
    auto *r = static_cast<XtPoolRing *>(h);
    if (!r || seq <= 0) return -2;
    const int64_t applied = __atomic_load_n(&r->words_host[1], __ATOMIC_ACQUIRE);
    if (seq - applied >= r->capacity) return -3;   // full
    int32_t *e = r->ring_host + (seq % r->capacity) * 4;
    e[1] = layer;
    e[2] = expert;
    e[3] = slot;
    __atomic_store_n(&e[0], int32_t(uint32_t(seq & 0xFFFFFFFFll)), __ATOMIC_RELEASE);
    __atomic_store_n(&r->words_host[0], seq, __ATOMIC_RELEASE);
    return 0;
}

int64_t xt_pool_ring_applied(void *h) {
    auto *r = static_cast<XtPoolRing *>(h);
    return r ? __atomic_load_n(&r->words_host[1], __ATOMIC_ACQUIRE) : -1;
}

int xt_pool_ring_commit(void *h, int32_t *const *tables, int n_tables, int *error, cudaStream_t stream) {
    auto *r = static_cast<XtPoolRing *>(h);
    if (!r || n_tables <= 0) return -2;
    const cudaError_t e = xt_launch(pool_commit_kernel, dim3(1), dim3(32), 0, stream,
                                    static_cast<const volatile int32_t *>(r->ring_dev),
                                    static_cast<const volatile int64_t *>(r->words_dev), r->capacity, r->state,
                                    tables, n_tables, static_cast<volatile int64_t *>(r->words_dev + 1), error);
    return e == cudaSuccess ? 0 : -1;
}

int xt_pool_ring_landed(void *h, int64_t seq, cudaStream_t stream) {
    auto *r = static_cast<XtPoolRing *>(h);
    if (!r) return -2;
    pool_landed_kernel<<<1, 32, 0, stream>>>(r->state, seq);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
