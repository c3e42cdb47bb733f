// Virtual-memory arenas for elastic expert slots: a fixed device address range is reserved once, and physical memory
// is mapped into it and released again granule by granule (cuMemAddressReserve / cuMemCreate / cuMemMap /
// cuMemSetAccess / cuMemUnmap / cuMemRelease). Tensors and captured CUDA graphs keep the arena's base pointer for good;
// only the physical backing of its tail comes and goes. The driver functions are fetched through
// cudaGetDriverEntryPoint, so the library links only the runtime.
// Reference parity: csrc/mailbox/mailbox.cpp:754-1180 (xtier_mailbox_vmm_*: reserve, map, unmap of arena granules).
// The arena bookkeeping (one handle per granule, prefix-mapped ranges) is this project's own.
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <vector>

namespace {

using PFN_reserve = CUresult (*)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long);
using PFN_free_va = CUresult (*)(CUdeviceptr, size_t);
using PFN_create = CUresult (*)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                                unsigned long long);
using PFN_release = CUresult (*)(CUmemGenericAllocationHandle);
using PFN_map = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
using PFN_unmap = CUresult (*)(CUdeviceptr, size_t);
using PFN_access = CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t);
using PFN_gran = CUresult (*)(size_t *, const CUmemAllocationProp *, CUmemAllocationGranularity_flags);

struct Driver {
    PFN_reserve reserve = nullptr;
    PFN_free_va free_va = nullptr;
    PFN_create create = nullptr;
    PFN_release release = nullptr;
    PFN_map map = nullptr;
    PFN_unmap unmap = nullptr;
    PFN_access access = nullptr;
    PFN_gran gran = nullptr;
    bool ok = false;
};

template <class F>
bool entry(const char *name, F &fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return false;
    fn = reinterpret_cast<F>(p);
    return p != nullptr;
}

Driver &driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        d.ok = entry("cuMemAddressReserve", d.reserve) && entry("cuMemAddressFree", d.free_va) &&
               entry("cuMemCreate", d.create) && entry("cuMemRelease", d.release) && entry("cuMemMap", d.map) &&
               entry("cuMemUnmap", d.unmap) && entry("cuMemSetAccess", d.access) &&
               entry("cuMemGetAllocationGranularity", d.gran);
    });
    return d;
}

struct Arena {
    int device;
    size_t bytes, granule;
    std::vector<CUmemGenericAllocationHandle> handles;   // per granule; 0: not mapped
};

std::mutex g_mu;
std::map<CUdeviceptr, Arena> g_arenas;

CUmemAllocationProp prop_of(int device) {
    CUmemAllocationProp p = {};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = device;
    return p;
}

}  // namespace

extern "C" {

// Minimum mapping granularity of `device` (bytes), 0 when the driver lacks the VMM calls.
size_t xt_vmm_granularity(int device) {
    Driver &d = driver();
    if (!d.ok) return 0;
    CUmemAllocationProp p = prop_of(device);
    size_t g = 0;
    if (d.gran(&g, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM) != CUDA_SUCCESS) return 0;
    return g;
}

// Reserves `bytes` (rounded up to the granularity) of device address space; *base receives it. 0 or an error code.
int xt_vmm_reserve(int device, size_t bytes, void **base, size_t *reserved) {
    Driver &d = driver();
    if (!d.ok) return -1;
    const size_t g = xt_vmm_granularity(device);
    if (!g || !bytes) return -2;
    const size_t n = (bytes + g - 1) / g * g;
    CUdeviceptr va = 0;
    CUresult r = d.reserve(&va, n, g, 0, 0);
    if (r != CUDA_SUCCESS) return int(r);
    std::lock_guard<std::mutex> lk(g_mu);
    g_arenas[va] = Arena{device, n, g, std::vector<CUmemGenericAllocationHandle>(n / g, 0)};
    *base = reinterpret_cast<void *>(va);
    *reserved = n;
    return 0;
}

// Makes granules [g0, g1) of the arena at `base` backed by device memory readable and writable from its device.
// Granules already mapped are kept. On failure, the granules this call mapped are released again.
int xt_vmm_map(void *base, size_t g0, size_t g1) {
    Driver &d = driver();
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_arenas.find(reinterpret_cast<CUdeviceptr>(base));
    if (it == g_arenas.end()) return -1;
    Arena &a = it->second;
    if (g0 > g1 || g1 > a.handles.size()) return -2;
    CUmemAllocationProp p = prop_of(a.device);
    CUmemAccessDesc acc = {};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = a.device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    std::vector<size_t> done;
    for (size_t i = g0; i < g1; ++i) {
        if (a.handles[i]) continue;
        const CUdeviceptr at = it->first + i * a.granule;
        CUmemGenericAllocationHandle h = 0;
        CUresult r = d.create(&h, a.granule, &p, 0);
        if (r == CUDA_SUCCESS) {
            r = d.map(at, a.granule, 0, h, 0);
            if (r == CUDA_SUCCESS) {
                r = d.access(at, a.granule, &acc, 1);
                if (r != CUDA_SUCCESS) d.unmap(at, a.granule);
            }
            if (r != CUDA_SUCCESS) d.release(h);
        }
        if (r != CUDA_SUCCESS) {
            for (size_t j : done) {
                d.unmap(it->first + j * a.granule, a.granule);
                d.release(a.handles[j]);
                a.handles[j] = 0;
            }
            return int(r);
        }
        a.handles[i] = h;
        done.push_back(i);
    }
    return 0;
}

// Unmaps granules [g0, g1) and gives their memory back. The caller guarantees that no queued or running kernel reads
// them (the device was synchronized after the last reader was unpublished).
int xt_vmm_unmap(void *base, size_t g0, size_t g1) {
    Driver &d = driver();
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_arenas.find(reinterpret_cast<CUdeviceptr>(base));
    if (it == g_arenas.end()) return -1;
    Arena &a = it->second;
    if (g0 > g1 || g1 > a.handles.size()) return -2;
    int rc = 0;
    for (size_t i = g0; i < g1; ++i) {
        if (!a.handles[i]) continue;
        CUresult r = d.unmap(it->first + i * a.granule, a.granule);
        if (r == CUDA_SUCCESS) r = d.release(a.handles[i]);
        if (r != CUDA_SUCCESS) rc = int(r);
        a.handles[i] = 0;
    }
    return rc;
}

// Number of mapped granules of the arena (-1: unknown arena).
long long xt_vmm_mapped(void *base) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_arenas.find(reinterpret_cast<CUdeviceptr>(base));
    if (it == g_arenas.end()) return -1;
    long long n = 0;
    for (auto h : it->second.handles) n += h != 0;
    return n;
}

// Unmaps everything and frees the address range.
int xt_vmm_free(void *base) {
    Driver &d = driver();
    size_t n;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_arenas.find(reinterpret_cast<CUdeviceptr>(base));
        if (it == g_arenas.end()) return -1;
        n = it->second.handles.size();
    }
    int rc = xt_vmm_unmap(base, 0, n);
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_arenas.find(reinterpret_cast<CUdeviceptr>(base));
    CUresult r = d.free_va(it->first, it->second.bytes);
    g_arenas.erase(it);
    return rc ? rc : int(r);
}

}  // extern "C"
