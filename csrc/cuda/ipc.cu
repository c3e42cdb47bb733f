// Peer memory plumbing for the in-kernel NVLink paths: export / import CUDA IPC handles of device buffers, so that every
// rank maps every peer's buffer and kernels can load from and store to it directly (plain ld/st over NVLink; no TMA
// multicast is ever issued on peer memory). The handle bytes travel between processes through torch.distributed.
#include <cuda_runtime.h>
#include <string.h>

extern "C" {

// Writes the 64-byte IPC handle of the allocation containing `ptr` into out. 0 or a CUDA error code.
int xt_ipc_export(void *ptr, void *out) {
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) return int(e);
    memcpy(out, &h, sizeof h);
    return 0;
}

// Maps a peer's allocation; *ptr receives its address in this process. 0 or a CUDA error code.
int xt_ipc_open(const void *handle, void **ptr) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return int(e);
}

int xt_ipc_close(void *ptr) { return int(cudaIpcCloseMemHandle(ptr)); }

int xt_ipc_handle_bytes(void) { return int(sizeof(cudaIpcMemHandle_t)); }

// 1 when this device can access `peer` directly (NVLink / PCIe P2P).
int xt_can_access_peer(int dev, int peer) {
    int ok = 0;
    cudaDeviceCanAccessPeer(&ok, dev, peer);
    return ok;
}

}  // extern "C"

extern "C" {

// A dedicated zeroed device allocation for a symmetric buffer (its IPC handle then names exactly this buffer).
int xt_ipc_alloc(size_t bytes, void **ptr) {
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) return int(e);
    e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return int(e);
}

int xt_ipc_free(void *ptr) { return int(cudaFree(ptr)); }

}  // extern "C"

extern "C" {

// 1 when `ptr` is page-locked host memory that kernels can read through the same address (mapped under unified
// addressing), else 0: the check before a kernel is given a host pointer.
int xt_host_ptr_mapped(const void *ptr) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return (a.type == cudaMemoryTypeHost && a.devicePointer == ptr) ? 1 : 0;
}

// Page-locks host memory another allocator owns (the CPU engine's weight shards) and maps it for kernels: *dev is the
// address kernels read it through. 0 or the CUDA error code (nothing stays registered on an error).
int xt_host_register_mapped(void *ptr, size_t bytes, void **dev) {
    cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return int(e);
    }
    e = cudaHostGetDevicePointer(dev, ptr, 0);
    if (e != cudaSuccess) {
        cudaHostUnregister(ptr);
        cudaGetLastError();
        return int(e);
    }
    return 0;
}

int xt_host_unregister(void *ptr) {
    const cudaError_t e = cudaHostUnregister(ptr);
    if (e != cudaSuccess) cudaGetLastError();
    return int(e);
}

}  // extern "C"
