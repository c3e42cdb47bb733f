// CPU<->GPU mailbox: the layout both sides agree on (device kernels in csrc/cuda/moe_decode.cu, host dispatcher in
// csrc/mailbox/mailbox.cpp).
//
// A mailbox slot lives in mapped pinned host memory (cudaHostAllocMapped). A decode MoE call on the GPU writes the
// token activations, the routes the CPU must compute (id or -1) and their weights into the slot, then publishes a new
// sequence number in `req` with a system-scope release store. The dispatcher thread polls `req`, runs the CPU engine of
// `layer` straight into the slot's `y`, and publishes the same number in `resp`. The GPU side waits for `resp` with a
// deadline (globaltimer), so a CPU that never answers makes the call fail with an error word instead of hanging the GPU.
// The sequence counter lives in device memory, so replays of a captured CUDA graph need no host involvement.
#pragma once
#include <stdint.h>

#define XT_MB_MAX_TOKENS 32
#define XT_MB_MAX_ROUTES 16   // per token (top-k plus shared experts)

struct XtMailboxHeader {
    volatile uint32_t req;        // GPU -> CPU: sequence of the newest request
    uint32_t pad0[31];
    volatile uint32_t resp;       // CPU -> GPU: sequence of the newest answered request
    uint32_t pad1[31];
    volatile int32_t layer, m, k, hidden;   // request fields, written before req
    volatile uint32_t gpu_error;  // GPU -> host: 1 = a wait timed out
    volatile uint32_t cpu_error;  // CPU -> host: 1 = an engine call failed
    uint32_t pad2[26];
};

// Device-resident state of one mailbox slot.
struct XtMailboxDev {
    uint32_t seq;       // last published sequence
    uint32_t pending;   // 1 when the last call has a CPU part to wait for
    uint32_t any;       // accumulates "some route goes to the CPU" during a call
    uint32_t done;      // CTAs finished writing the current request
    uint32_t error;     // 1 = a wait timed out (sticky until the host clears it)
    uint32_t pad[3];
};

// Everything a kernel needs to use a slot (device-visible addresses).
struct XtMailbox {
    XtMailboxHeader *hdr;     // mapped host
    uint16_t *x;              // [max_tokens, hidden] bf16 bits
    int32_t *ids;             // [max_tokens, max_routes]
    float *w;                 // [max_tokens, max_routes]
    int32_t *orig;            // [max_tokens, max_routes] routes as routed (statistics / adaptive policy)
    float *y;                 // [max_tokens, hidden] CPU result
    XtMailboxDev *dev;        // device memory
    unsigned long long timeout_ns;
};

// Host-side offsets of the arrays inside one slot allocation.
static inline unsigned long long xt_mb_bytes(int hidden) {
    unsigned long long b = sizeof(XtMailboxHeader);
    b += 2ull * XT_MB_MAX_TOKENS * hidden;                   // x
    b += 3ull * 4 * XT_MB_MAX_TOKENS * XT_MB_MAX_ROUTES;     // ids, w, orig
    b = (b + 255) & ~255ull;
    b += 4ull * XT_MB_MAX_TOKENS * hidden;                   // y
    return b;
}
