// Shared device helpers of the sm_100a kernels (B200 only: compiled with -gencode arch=compute_100a,code=sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define XT_DEV __device__ __forceinline__

#include <stdlib.h>
#include <mutex>
#include <utility>

namespace xt {

// Programmatic dependent launch (PDL). A kernel started by xt_launch may begin while its predecessor in the stream
// still runs: before pdl_wait() it may only read data no earlier kernel writes (weights); pdl_wait() returns once the
// predecessor grid has completed and its memory is visible (a no-op for a kernel launched without the attribute);
// pdl_trigger() lets the successor start launching. Every kernel launched by xt_launch calls pdl_wait() before its
// first dependent read and before any global write, so a chain of such kernels stays ordered.
XT_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
XT_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

inline bool pdl_enabled() {   // XTIER_PDL=0 turns the overlap off
    static const bool on = [] {
        const char *v = getenv("XTIER_PDL");
        return !v || atoi(v) != 0;
    }();
    return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t xt_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Opts a kernel into `bytes` of dynamic shared memory on the current device. The attribute belongs to the device's
// context, so a process that drives several GPUs must set it once per device: the flag kept here is a bit per device
// (devices 0-63) per kernel, and a device beyond that sets the attribute on every call.
inline cudaError_t xt_smem_optin(const void *func, int bytes) {
    struct Entry { const void *f; int bytes; uint64_t devs; };
    static Entry table[256];
    static int used = 0;
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    Entry *hit = nullptr;
    for (int i = 0; i < used; ++i)
        if (table[i].f == func && table[i].bytes == bytes) hit = &table[i];
    if (hit && dev < 64 && (hit->devs >> dev & 1)) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    if (!hit && used < 256) hit = &table[used++], *hit = Entry{func, bytes, 0};
    if (hit && dev < 64) hit->devs |= uint64_t(1) << dev;
    return cudaSuccess;
}

template <typename... KArgs>
inline cudaError_t xt_smem_optin(void (*kernel)(KArgs...), int bytes) {
    return xt_smem_optin(reinterpret_cast<const void *>(kernel), bytes);
}

XT_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

XT_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over groups of L consecutive lanes (L a power of two <= 32); every lane of a group gets the group's sum.
template <int L>
XT_DEV float group_sum(float v) {
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Four E2M1 pairs (one 32-bit word, byte i = elements 2i and 2i+1, low nibble first) -> four f16x2, using the
// hardware conversion of sm_100 (cvt.rn.f16x2.e2m1x2 puts the low nibble in the low half).
XT_DEV void e2m1x8_to_h2(uint32_t w, __half2 (&out)[4]) {
    uint32_t r0, r1, r2, r3;
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
        : "r"(w));
    out[0] = *reinterpret_cast<__half2 *>(&r0);
    out[1] = *reinterpret_cast<__half2 *>(&r1);
    out[2] = *reinterpret_cast<__half2 *>(&r2);
    out[3] = *reinterpret_cast<__half2 *>(&r3);
}

// Two E4M3 bytes (low byte first) -> two floats (hardware conversion through f16x2)
XT_DEV float2 e4m3x2_to_f2(uint16_t v) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(r) : "h"(v));
    return __half22float2(*reinterpret_cast<__half2 *>(&r));
}

XT_DEV float e4m3_to_f(uint8_t b) { return e4m3x2_to_f2(uint16_t(b)).x; }

// Two E4M3 bytes (low byte first) -> f16 pair (exact: every E4M3 value is an f16 value)
XT_DEV __half2 e4m3x2_to_h2(uint16_t v) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(r) : "h"(v));
    return *reinterpret_cast<__half2 *>(&r);
}

// 2^x, hardware approximation (results below 2^-126 flush to zero)
XT_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

XT_DEV float ue8m0_to_f(uint8_t b) { return b ? __uint_as_float(uint32_t(b) << 23) : 5.877471754e-39f; }

XT_DEV uint4 ldg_nc_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// System-scope acquire load / release store (mapped host memory shared with the CPU).
XT_DEV uint32_t ld_acquire_sys(const volatile uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

XT_DEV void st_release_sys(volatile uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

XT_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
    return t;
}

// float -> E4M3 byte (round to nearest even, saturating at 448)
XT_DEV uint8_t f32_to_e4m3(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(0.f), "f"(v));
    return uint8_t(r & 0xFF);
}

// two floats -> one byte of two E2M1 codes (a in the low nibble), round to nearest even, saturating at 6
XT_DEV uint8_t f32x2_to_e2m1(float a, float b) {
    uint16_t r;
    asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n cvt.u16.u8 %0, t;\n}\n" : "=h"(r) : "f"(a), "f"(b));
    return uint8_t(r);
}

XT_DEV float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace xt
