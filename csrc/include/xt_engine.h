// CPU expert engine and cold-expert store: C ABI (loaded with ctypes by xtier_b200.engine).
//
// Routed-expert MoE on the CPU for tokens whose experts are not in a GPU hot slot. Weights are FP4 (E2M1, two per byte,
// even element in the low nibble) with NVFP4 (E4M3 per 16 + FP32 globals) or MXFP4 (UE8M0 per 32) block scales, in the
// layout of the checkpoints:
//   w13 [n, 2I, H/2] gate rows then up rows   s13 [n, 2I, H/bs]   g13 [n, 2]
//   w2  [n, H, I/2]                           s2  [n, H, I/bs]    g2  [n]
// where n = slots + shared. Experts 0..experts-1 are routed; `shared` extra experts (the arrays' last entries) are applied
// to every token with weight 1. Activations are BF16 bits, outputs FP32; the intermediate stays FP32 (the down
// projection consumes it as an exact hi+lo BF16 pair on AVX-512, FP32 elsewhere). Results do not depend on the thread
// count: every output element is summed by one task in a fixed order (expert id ascending, then the shared experts).
//
// Reference parity: csrc/include/xtier_engine.h:31-123 (create3/4, forward, forward_decode, place, slot pin/unpin,
// slot table, slot pieces, set_swiglu, shape, read_probe, tail stats, last timings, shard, nodes, worker cpus, isa,
// destroy) and :125-147 (cold store). The function set is kept because the planner probe, the cold store and the tools
// drive the engine through it; names, argument order and internals are this project's own.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// fmt: 0 = NVFP4, 1 = MXFP4. limit > 0 clamps up to [-L, L] and gate to (-inf, L] before SiLU. threads: workers of the
// process-wide pool (0: all allowed CPUs). slots: RAM slots for routed experts (== experts when nothing is cold);
// resident[j] is the expert held by slot j (-1 empty; NULL means slot j holds expert j). With w13 == NULL the shards are
// allocated but not filled (the caller writes them through xt_engine_slot_pieces). Returns NULL on error.
void *xt_engine_create(int hidden, int inter, int experts, int shared, int slots, int threads, float limit, int fmt,
                       const uint8_t *w13, const uint8_t *w2, const uint8_t *s13, const uint8_t *s2, const float *g13,
                       const float *g2, const int32_t *resident);
void xt_engine_destroy(void *plan);
// GPT-OSS form gate*sigmoid(alpha*gate)*(up+beta) (defaults 1, 0: plain SiLU).
int xt_engine_set_swiglu(void *plan, float alpha, float beta);
// x: BF16 [m, H]; ids int32 [m, k] (-1: skip, e.g. a route served on the GPU); w float [m, k]; y float [m, H]
// (overwritten). Returns the number of expert groups computed, or -1 (xt_engine_error).
int xt_engine_forward(void *plan, int m, int k, const uint16_t *x, const int32_t *ids, const float *w, float *y);
// The decode path: as forward, plus XTIER_TAIL_SKIP and the route trace hook.
int xt_engine_forward_decode(void *plan, int m, int k, const uint16_t *x, const int32_t *ids, const float *w, float *y);
// Streams the routed bytes without computing (memory ceiling of the kernels); y untouched.
int xt_engine_read_probe(void *plan, int m, int k, const int32_t *ids);
// [hidden, inter, experts, shared, slots, nodes, threads]
int xt_engine_shape(void *plan, int *out7);
// Two wall-clock durations of the last forward in microseconds: gate/up phase, down phase.
void xt_engine_last_timings(void *plan, double *out2);
// out[3]: decode calls tail skip looked at, distinct experts, experts left out.
void xt_engine_tail_stats(void *plan, double *out3);
// Slot of every routed expert (-1 if not in RAM): table[experts]. Returns slots.
int xt_engine_slot_table(void *plan, int32_t *table);
// Mark `expert` as held by `slot` after its weights were written there (expert -1: the slot holds nothing). Returns
// the previous expert of the slot or -1;
// -2 bad arguments, -3 a forward in progress.
int xt_engine_place(void *plan, int expert, int slot);
// Global scales of every routed expert (g13 [E, 2], g2 [E]); from then on a slot takes the scales of the expert placed
// or read into it (cold reads, place). Returns 0, -1 on bad arguments, -3 while a forward runs.
int xt_engine_expert_scales(void *plan, const float *g13, const float *g2);
// Pin the slot holding `expert` against eviction while another thread reads it (-1: not in RAM).
int xt_engine_slot_pin(void *plan, int expert);
void xt_engine_slot_unpin(void *plan, int slot);
// Six pieces of a slot on worker node `node`: gate, up, gate scales, up scales, down, down scales. 0 or -1.
int xt_engine_slot_pieces(void *plan, int slot, int node, void **ptrs, size_t *bytes);
int xt_engine_nodes(void *plan);
// The whole shard of worker node `node`: base address and bytes (every slot, routed and shared), the bytes between two
// slots, and the six pieces' offsets inside a slot and sizes. 0 or -1.
int xt_engine_shard(void *plan, int node, void **base, size_t *bytes, size_t *stride, size_t *piece_off,
                    size_t *piece_bytes);
// Cold experts: forward reads experts that are not in a RAM slot from the store before computing them.
// files/offsets [experts * nodes]: record of expert e's node part n (file -1: never cold). scores: initial use counts.
int xt_engine_cold_attach(void *plan, void *store, const int32_t *files, const long long *offsets, const float *scores,
                          float half_life);
// The same with one location per piece: files / offsets [experts * nodes * 6] (pieces of a record may sit on different
// drives, e.g. records split into units).
int xt_engine_cold_attach_pieces(void *plan, void *store, const int32_t *files, const long long *offsets,
                                 const float *scores, float half_life);
// out[4]: forwards, experts read from NVMe, seconds waited for reads, decode forwards.
void xt_engine_cold_stats(void *plan, double *out4);
// CPUs the workers would bind to for `threads`.
int xt_engine_worker_cpus(int threads, int *cpus, int capacity);
const char *xt_engine_isa(void);
const char *xt_engine_error(void);

// Cold store: one file per drive, O_DIRECT both ways. Offsets and piece sizes are multiples of 512 bytes, read buffers
// 512-aligned. NULL on error.
void *xt_cold_open(const char *const *paths, int count, int threads, int writable);
int xt_cold_write(void *store, int file, long long offset, const void *const *pieces, const size_t *sizes, int n);
// jobs reads at once: job j reads n pieces from files[j] at offsets[j] into dst[j*n ..], sizes[j*n ..]. 0 or -1.
int xt_cold_read(void *store, int jobs, const int *files, const long long *offsets, void *const *dst,
                 const size_t *sizes, int n);
// Asynchronous: returns a ticket; xt_cold_wait waits for the jobs of groups [g0, g1).
void *xt_cold_submit(void *store, int jobs, const int *files, const long long *offsets, void *const *dst,
                     const size_t *sizes, int n, const int *groups, int group_count);
int xt_cold_wait(void *store, void *ticket, int g0, int g1);
int xt_cold_finish(void *store, void *ticket);
// out[4]: bytes read, bytes written, read jobs, seconds from submit to completion (summed).
void xt_cold_stats(void *store, double *out4);
void xt_cold_close(void *store);
const char *xt_cold_error(void);

#ifdef __cplusplus
}
#endif
