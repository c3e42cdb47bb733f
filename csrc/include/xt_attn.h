// C entry points of the decode attention that need no device allocation by the caller.
//
// xt_attn_decode_noalloc has no counterpart in the reference. It exists for callers that cannot call cudaMalloc:
// code that runs inside another framework's memory pool and has no allocator handed to it, plugins whose host
// process forbids device allocation after start-up, and serving loops that must never enter the driver's allocator
// while they run. Its split workspace is a fixed array in the library's device memory (the limits below), which
// every GPU that loads the library holds until the process exits.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// Floats of the fixed split workspace (2 MiB) and arrival counters of the fixed array.
#define XT_AD_NOALLOC_FLOATS (512 * 1024)
#define XT_AD_NOALLOC_COUNTERS 4096
// Return code of a call whose workspace would not fit in the fixed array.
#define XT_AD_NOALLOC_TOO_BIG (-6)

#ifdef __cplusplus
extern "C" {
#endif

// q [B, Hq, 128] bf16, k_cache / v_cache [B, Hkv, L, 128] bf16, seqlens [B] int32 (device), out [B, Hq, 128] bf16;
// all device pointers on the current device; Hq / Hkv must be 1, 2, 4, 8 or 16. Returns 0 on success; -2 for bad
// arguments (nothing is enqueued); XT_AD_NOALLOC_TOO_BIG when B * Hkv * splits * (Hq / Hkv) * 130 floats or B * Hkv
// counters exceed the fixed array (nothing is enqueued); a positive CUDA error code from the once-per-device set-up;
// -1 when the launch failed. The first call on a device performs the set-up: make it before any stream capture.
// Calls share one array: calls that overlap on the GPU race and must be serialized by the caller.
int xt_attn_decode_noalloc(const void *q, const void *k_cache, const void *v_cache, const int32_t *seqlens, void *out,
                           int B, int Hq, int Hkv, int L, int splits, float scale, cudaStream_t stream);

// Text of the last error of xt_attn_decode_noalloc on the calling host thread.
const char *xt_attn_decode_noalloc_error(void);

// out[0] = floats of the split workspace, out[1] = arrival counters.
void xt_attn_decode_noalloc_limits(long long *out);

#ifdef __cplusplus
}
#endif
