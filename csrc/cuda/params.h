// Launch parameters of the sm_100a kernels and their C launchers: shared by the .cu files and the torch bindings.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../include/xt_mailbox.h"

namespace xt {

struct RouteParams {
    const __nv_bfloat16 *x;   // [m, H]
    const __nv_bfloat16 *wr;  // [E, H] router weight
    const float *bias;        // [E] added to the logits before selection (may be null)
    const float *corr;        // [E] grouped mode: selection bias (e_score_correction_bias), may be null
    const int32_t *table;     // [E] residency: slot or -1 (null: expert id == slot, everything on the GPU)
    const int32_t *shared_slots;   // [n_shared]
    const int32_t *active;    // [m] token flags (may be null): a token with flag 0 skips its routed experts
    const float *logits_in;   // [m, E] precomputed FP32 router logits (prefill; may be null): selection only
    // miss share (may be null / 0): a token with at least share_min routes on the CPU tier sends its first one to the
    // GPU instead, which reads that expert from pinned host memory (slot = host_base + cold_index[expert])
    const int32_t *cold_index;
    int share_min, host_base;
    // PCIe staging (may be null / 0; expert parallelism): a CPU-tier route whose expert has a host copy the GPU can
    // read (cold_index >= 0) claims one of stage_max staging slots and becomes GPU slot stage_slot0 + index. claim [E]
    // (-1 free, -2 being claimed, -3 no room, else the staging index), claim_list [E] (the experts in claim order),
    // claim_count [1]; the staging copy kernel reads them and resets them for the next call
    int32_t *claim, *claim_list, *claim_count;
    int stage_max, stage_slot0;
    int32_t *ids;             // [m, kk] original expert ids (-1 for shared)
    float *w;                 // [m, kk]
    int32_t *slots;           // [m, kk] GPU slot or -1
    float *ws_logits;         // [m, E] scratch: router logits of the call
    uint32_t *ws_count;       // [m] scratch: CTAs done per token (zero before the first call; reset by the kernel)
    int m, H, E, k, n_shared, mode, n_group, topk_group, renorm, layer;
    float scale;
};

struct GateUpParams {
    const __nv_bfloat16 *x;   // [m, H]
    const int32_t *slots;     // [m, kk]
    const uint8_t *w13;       // [S, 2I, H/2]
    const uint8_t *s13;       // [S, 2I, H/bs]
    const float *g13;         // [S, 2]
    __half *mid;              // [m*kk, I] f16 (the down kernel's FP4 x f16 products take it as is)
    int routes, kk, H, I, fmt;
    float limit, alpha, beta;
    // slot pools of the peer GPUs (may be null): [W][6] base addresses (w13, s13, g13, w2, s2, g2) of every rank's
    // pool; a slot then names rank slot / spr, local slot slot % spr, read over NVLink when the rank is another GPU
    const unsigned long long *peer;
    int spr;
    // pinned host pool of the CPU tier's experts (may be null): [6] base addresses (w13, s13, g13, w2, s2, g2); a slot
    // >= host_base names host expert slot - host_base, read over PCIe
    const unsigned long long *host;
    int host_base;
};

struct DownParams {
    const __half *mid;        // [m*kk, I] f16
    const int32_t *slots;     // [m, kk]
    const float *w;           // [m, kk]
    const uint8_t *w2;        // [S, H, I/2]
    const uint8_t *s2;        // [S, H, I/bs]
    const float *g2;          // [S]
    const __nv_bfloat16 *add; // [m, H] optional extra term (e.g. a shared expert computed elsewhere), may be null
    __nv_bfloat16 *out;       // [m, H]
    float *out_f32;           // [m, H] optional FP32 copy of the GPU part (tests), may be null
    float *gpu_part;          // [m, H] scratch: the GPU part while a CPU part is pending (mailbox calls)
    int kk, H, I, fmt;
    const unsigned long long *peer;   // as in GateUpParams (may be null)
    int spr;
    const unsigned long long *host;   // as in GateUpParams (may be null)
    int host_base;
};

struct RopeParams {
    const __nv_bfloat16 *qkv;   // [T, (Hq + 2 Hkv) * D]
    const __nv_bfloat16 *qn;    // [D] or null
    const __nv_bfloat16 *kn;    // [D] or null
    const int32_t *pos;         // [T]
    const int32_t *batch;       // [T] cache row of each token
    const int32_t *slot;        // [T] cache position of each token, or null: its RoPE position (tree drafts: nodes
                                // at the same depth share a position, each has its own slot)
    __nv_bfloat16 *q;           // [T, Hq, D]
    __nv_bfloat16 *kc, *vc;     // [B, Hkv, L, D]
    int T, Hq, Hkv, D, L;
    float theta, eps;
};

struct AttnDecodeParams {
    const __nv_bfloat16 *q;     // [B, Hq, D]
    const __nv_bfloat16 *kc;    // [B, Hkv, L, D]
    const __nv_bfloat16 *vc;
    const int32_t *seqlens;     // [B] keys to attend (including the current token)
    __nv_bfloat16 *out;         // [B, Hq, D]
    float *ws_o;                // [B, Hkv, S, G, D]
    float *ws_ml;               // [B, Hkv, S, G, 2]
    uint32_t *counters;         // [B, Hkv], zero before the first launch; the merging CTA resets its entry
    int Hq, Hkv, L, splits;
    float scale_log2;           // softmax scale * log2(e)
};

}  // namespace xt

extern "C" {
int xt_add_rmsnorm(const void *x, void *residual, const void *w, void *out, int T, int H, float eps,
                   cudaStream_t stream);
int xt_qk_norm_rope_kv(const xt::RopeParams *p, cudaStream_t stream);
int xt_attn_decode(const xt::AttnDecodeParams *p, int B, cudaStream_t stream);
int xt_moe_route(const xt::RouteParams *p, const XtMailbox *mb, int use_mb, cudaStream_t stream);
int xt_moe_gate_up(const xt::GateUpParams *p, cudaStream_t stream);
int xt_moe_down(const xt::DownParams *p, const XtMailbox *mb, int use_mb, int m, cudaStream_t stream);
int xt_gemm_tc(const void *A, const void *B, void *D, const void *R, int M, int N, int K, int *error,
               cudaStream_t stream);
int xt_gemm_tc_f32(const void *A, const void *B, float *D, int M, int N, int K, int *error, cudaStream_t stream);
int xt_gemv_bf16(const void *x, const void *W, const void *add, void *y, int m, int N, int K, cudaStream_t stream);
int xt_mx_quant_rows(const void *x, const int32_t *src, int R, int K, void *x8, void *sfx, cudaStream_t stream);
int xt_moe_grouped_mx(const void *x8, const void *sfx, int R, const void *codes, const void *scales, int slots,
                      const int32_t *tiles, int T, int gate_up, int K, int N_rows, int I, const float *gscale,
                      const float *route_w, const int32_t *dst_row, void *mid, float *y, int out_cols, int *error,
                      cudaStream_t stream);
void *xt_pool_ring_create(int capacity);
void xt_pool_ring_destroy(void *h);
int xt_pool_ring_post(void *h, int64_t seq, int layer, int expert, int slot);
int64_t xt_pool_ring_applied(void *h);
int xt_pool_ring_commit(void *h, int32_t *const *tables, int n_tables, int *error, cudaStream_t stream);
int xt_pool_ring_landed(void *h, int64_t seq, cudaStream_t stream);
int xt_skinny_splits(int N, int K, int sms);
int xt_skinny_gemm(const void *x, const void *W, const void *add, void *y, float *part, int M, int N, int K,
                   int splits, int *error, cudaStream_t stream);
int xt_fp8_rows(const void *tab, const void *sc, const int64_t *ids, long long lo, long long hi, int n, int dim,
                int blk, void *out, cudaStream_t stream);
int xt_gemv_fp8(const void *x, const void *W, const float *S, const void *add, void *y, int m, int N, int K,
                cudaStream_t stream);
int xt_fp8_dequant(const void *W, const float *S, void *out, int N, int K, cudaStream_t stream);
int xt_spec_truncate(float *q, const int64_t *tokens, const int32_t *topk, int32_t *flags, float th,
                     long long stride_b, long long stride_s, int B, int S, int V, cudaStream_t stream);
}

namespace xt {
// Expert-parallel MoE over symmetric peer memory (csrc/cuda/moe_decode.cu, ep_* kernels). Every rank holds the same
// buffer layout; peer[r] is rank r's buffer as mapped in this process.
//   rx    [W src][R][H] bf16     tokens received from each source rank
//   meta  [W src][R] int4        {local expert, source token, source route, weight bits}
//   cnt   [W src] int32 (128 B apart)   routes received from each source
//   flag  [W src] uint32 (128 B apart)  epoch of the source's last dispatch into this buffer
//   ret   [T*k][H] fp32          weighted expert outputs of this rank's own routes, written by the owner ranks
//   rflag [W dst] uint32 (128 B apart)  epoch of the owner rank's last return into this buffer
struct EpParams {
    int W, rank, E, El, H, I, k, T, R, fmt;
    const uint64_t *peer;        // [W] device array
    size_t off_rx, off_meta, off_cnt, off_flag, off_ret, off_rflag;
    const __nv_bfloat16 *x;      // [T, H]
    const int32_t *ids;          // [T, k] global expert ids
    const float *w;              // [T, k]
    uint32_t *state;             // local: [0] epoch, [1] dispatch arrivals, [8 + s] down-send progress per source
    __half *mid;                 // local scratch [W*R, I] f16 (SwiGLU output)
    const uint8_t *w13, *s13, *w2, *s2;   // this rank's El experts
    const float *g13, *g2;
    const __nv_bfloat16 *add;    // [T, H] extra term of the combine (shared experts), may be null
    __nv_bfloat16 *out;          // [T, H]
    unsigned long long timeout_ns;
    int *error;
    // tiers (may be null / 0): slots [T, k] as the router wrote them -- rank * El + slot in the owner's GPU pool, or
    // -1 for a route the CPU tier computes; such routes are not dispatched, and the combine adds the mailbox's CPU
    // rows (a bounded wait for the dispatcher's answer) instead
    const int32_t *slots;
    XtMailbox mb;
    int use_mb;
    int by_expert;   // expert streams visit the received routes grouped by pool slot (0: arrival order)
    // PCIe staging (may be null / 0): local slots >= stage_base name staging slot (slot - stage_base), whose weights
    // the staging copy kernel brought from host memory earlier in the same call
    const uint8_t *st_w13, *st_s13, *st_w2, *st_s2;
    const float *st_g13, *st_g2;
    int stage_base;
};

// The staging copy (csrc/cuda/ep_stage.cu): the experts the router claimed, from the CPU engine's host memory (mapped,
// read over PCIe) into the GPU staging slots. An engine slot keeps its expert as 6 pieces per NUMA node (gate codes,
// up codes, gate scales, up scales, down codes, down scales; node n holds rows [n*I/N, (n+1)*I/N) of gate and up and
// [n*H/N, (n+1)*H/N) of down).
struct StageParams {
    const int32_t *claim_list;   // [E]
    int32_t *claim;              // [E]
    int32_t *claim_count;        // [1]
    uint32_t *done;              // [1] CTAs finished (the last one resets the claims)
    const int32_t *cold_index;   // [E] engine slot of the expert, or -1
    unsigned long long base[8];  // device address of each node's shard
    unsigned long long stride;   // bytes per engine slot in a shard
    unsigned long long piece_off[6], piece_bytes[6];
    uint8_t *w13, *s13, *w2, *s2;   // staging [stage_max, ...] in the pool layout
    float *g13, *g2;                // [stage_max, 2], [stage_max]
    const float *src_g13, *src_g2;  // global scales by engine slot: [slots, 2], [slots]
    int nodes, stage_max, E, I, H, bs, chunks;
};

// Per-head small GEMM of the MLA decode step (csrc/cuda/mla_proj.cu).
struct HeadGemmParams {
    const __nv_bfloat16 *x;   // X[t, h, k] at x + t * xs_t + h * xs_h + k
    const __nv_bfloat16 *w;   // [heads, K, N]
    __nv_bfloat16 *y;         // Y[t, h, n] at y + t * ys_t + h * ys_h + n
    long long xs_t, xs_h, ys_t, ys_h;
    int T, K, N;
    // optional rotary part (rope_dims > 0): Y[t, h, rope_y + i] = NeoX rotation of X[t, h, rope_x + i]
    const int32_t *pos;
    int rope_x, rope_y, rope_dims;
    float theta;
};
}  // namespace xt

extern "C" int xt_ep_moe(const xt::EpParams *p, int phase, cudaStream_t stream);
extern "C" int xt_ep_stage(const xt::StageParams *p, cudaStream_t stream);
extern "C" int xt_qsa_kv_write(const void *x, const int64_t *slot, int T, int H, int D, void *codes, void *scales,
                               cudaStream_t stream);
extern "C" int xt_qsa_decode(const void *q, const int32_t *idx, int B, int nsel, int Hq, int Hkv, int D,
                             const void *kc, const void *ks, const void *vc, const void *vs, float *part_o,
                             float *part_ml, void *out, float scale, cudaStream_t stream);

namespace xt {
// Tensor-parallel GEMMs fused with their collective (csrc/cuda/gemm_tp.cu).
struct TpParams {
    int M, N, K, W, rank;
    const uint64_t *peer;       // [W] symmetric buffer bases (this process's mappings)
    size_t off_data[2];         // RS: receive region [W][M/W][N] bf16; AG: gather region [M][K] bf16 (per parity)
    size_t off_flags[2];        // RS: [W][tiles per owner] u32; AG: [M/128] u32 (per parity)
    uint32_t *state;            // local: [0] epoch, [1] arrivals of the reduce
    __nv_bfloat16 *out;         // RS: [M/W, N] reduced rows of this rank; AG: [M, N]
    const __nv_bfloat16 *residual;   // RS: [M/W, N] added to the reduced rows, may be null
    const __nv_bfloat16 *a_shard;    // AG push: [M/W, K]
    unsigned long long timeout_ns;
    int *error;
};
}  // namespace xt

extern "C" {
int xt_gemm_rs(const void *a, const void *b, const xt::TpParams *p, cudaStream_t stream);
int xt_ag_gemm(const void *b, const void *local_base, const xt::TpParams *p, cudaStream_t stream);
int xt_l2_prefetch(const uint64_t *ptrs, const uint64_t *bytes, int n, int ctas, cudaStream_t stream);
int xt_mla_kv_write(const void *lat, const int64_t *slot, void *codes, void *scales, void *rope, int T,
                    cudaStream_t stream);
int xt_dsa_key_write(const void *k, const int64_t *slot, void *codes, float *kscale, int T, cudaStream_t stream);
int xt_dsa_index_decode(const void *q, const float *w, const void *codes, const float *kscale, const int64_t *base,
                        const int32_t *len, float *scores, int Q, int max_len, cudaStream_t stream);
int xt_dsa_index_tc(const void *q8, const float *w, const void *codes, int64_t slots, const float *kscale,
                    const int64_t *base, const int32_t *len, float *scores, int Q, int max_len, int nq, int *error,
                    cudaStream_t stream);
int xt_topk_rows(const float *scores, int rows, int n, int K, const int32_t *len, int32_t *out, cudaStream_t stream);
int xt_dsa_quant_q(const void *q, const void *w, float w_scale, void *q8, float *w8, int rows, cudaStream_t stream);
int xt_rope_heads(const void *x, int64_t xs_t, int64_t xs_h, const int32_t *pos, float theta, void *y, int64_t ys_t,
                  int64_t ys_h, int T, int H, int d, cudaStream_t stream);
int xt_dsa_index_pf(const void *q8, const float *w, const void *codes, int64_t slots, const float *kscale,
                    int64_t row_base, const int32_t *len, float *scores, int Q, int max_len, int splits, int *error,
                    cudaStream_t stream);
int xt_moe_grouped(const void *x, int R, const void *codes, int slots, const int32_t *tiles, int T, int gate_up,
                   int K, int N_rows, int I, int fmt, const void *scales, const float *gscale, const float *route_w,
                   const int32_t *dst_row,
                   void *mid, float *y, int out_cols, int *error, cudaStream_t stream);
int xt_gather_rows(const void *x, const int32_t *src, void *X, int R, int H, cudaStream_t stream);
int xt_route_combine(const float *Ya, const int32_t *da, int ka, const float *Yb, const int32_t *db, int kb,
                     const void *add, void *out, int out_f32, int m, int H, cudaStream_t stream);
int xt_mla_prep(const void *in, int ld, int q_lora, const void *q_norm, const void *kv_norm, const int32_t *pos,
                const int64_t *slot, float eps, float theta, void *q_out, void *codes, void *scales, void *rope,
                void *lat_out, int T, cudaStream_t stream);
int xt_head_gemm(const xt::HeadGemmParams *p, int heads, cudaStream_t stream);
int xt_silu_mul(const void *in, void *out, int T, int I, cudaStream_t stream);
int xt_mhc_post(const void *x, const void *res, const float *post, const float *comb, void *out, int M, int H,
                cudaStream_t stream);
int xt_wo_a(const void *o, int64_t o_st, int64_t o_sg, const void *w8, const void *wb, const float *scale,
            int s_stride, void *out, int64_t out_st, int64_t out_sg, int T, int G, int R, int D, cudaStream_t stream);
int xt_hc_mix(const void *x, const void *wd, const void *wu, float *acc, void *out, int rows, int hc, int hs, int L,
              cudaStream_t stream);
int xt_gemm_mx8(const void *x8, const void *sfx, int M, const void *w8, const void *sfw, int N, int K,
                const void *residual, void *y, int *error, cudaStream_t stream);
int xt_attn_prefill(const void *q, int64_t q_ts, int64_t q_hs, const void *k, const void *v, int64_t kv_rows,
                    int64_t kv_row0, int64_t kv_hs, int T, int start, int Hq, int Hkv, void *out, int64_t out_ts,
                    int64_t out_hs, float scale, const unsigned long long *tree_mask, int *error,
                    cudaStream_t stream);
int xt_mla_flash(const void *q_lat, int64_t ql_ts, int64_t ql_hs, const void *q_rope, int64_t qr_ts, int64_t qr_hs,
                 const int32_t *idx, int Q, int nsel, const void *codes, const void *scales, const void *rope,
                 float *part_o, float *part_ml, void *out, int64_t out_ts, int64_t out_hs, float scale, int splits,
                 int nslots, int *error, cudaStream_t stream);
int xt_mla_decode(const void *q, const int32_t *idx, int Q, int nsel, const void *codes, const void *scales,
                  const void *rope, void *Kg, void *Vt, float *part_o, float *part_ml, void *out, float scale,
                  int *error, cudaStream_t stream);
}

