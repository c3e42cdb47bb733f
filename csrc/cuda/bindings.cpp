// torch op registrations of the sm_100a kernels (namespace `xtier`). Every op writes into tensors the caller owns and
// allocates nothing, so the ops can be captured into CUDA graphs. Checks are done once per call on the host.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "params.h"

extern "C" int xt_mailbox_view(void *h, void *out);

namespace {

using at::Tensor;
using xt::AttnDecodeParams;
using xt::DownParams;
using xt::GateUpParams;
using xt::RopeParams;
using xt::RouteParams;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(bool ok, const char *what) { TORCH_CHECK(ok, "xtier: ", what); }

void check_rc(int rc, const char *op) { TORCH_CHECK(rc == 0, "xtier: ", op, " launch failed (code ", rc, ")"); }

template <typename T>
T *ptr(const Tensor &t) {
    return reinterpret_cast<T *>(t.data_ptr());
}

template <typename T>
T *optr(const std::optional<Tensor> &t) {
    return t.has_value() && t->defined() ? reinterpret_cast<T *>(t->data_ptr()) : nullptr;
}

void cuda_contig(const Tensor &t, const char *name) {
    TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "xtier: ", name, " must be a contiguous CUDA tensor");
}

XtMailbox mailbox_view(int64_t handle) {
    XtMailbox v{};
    if (handle) TORCH_CHECK(xt_mailbox_view(reinterpret_cast<void *>(handle), &v) > 0, "xtier: bad mailbox handle");
    return v;
}

void add_rmsnorm(const Tensor &x, const std::optional<Tensor> &residual, const Tensor &w, const Tensor &out,
                 double eps) {
    cuda_contig(x, "x");
    cuda_contig(out, "out");
    check(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "add_rmsnorm wants bf16");
    const int H = int(x.size(-1));
    const int T = int(x.numel() / H);
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_add_rmsnorm(x.data_ptr(), optr<void>(residual), w.data_ptr(), out.data_ptr(), T, H, float(eps),
                            stream()),
             "add_rmsnorm");
}

void qk_norm_rope_kv(const Tensor &qkv, const std::optional<Tensor> &qn, const std::optional<Tensor> &kn,
                     const Tensor &pos, const Tensor &batch, const Tensor &q, const Tensor &kc, const Tensor &vc,
                     int64_t hq, int64_t hkv, double theta, double eps, const std::optional<Tensor> &slots) {
    cuda_contig(qkv, "qkv");
    cuda_contig(kc, "k_cache");
    cuda_contig(vc, "v_cache");
    check(pos.scalar_type() == at::kInt && batch.scalar_type() == at::kInt, "positions and batch must be int32");
    RopeParams p{};
    p.qkv = ptr<const __nv_bfloat16>(qkv);
    p.qn = optr<const __nv_bfloat16>(qn);
    p.kn = optr<const __nv_bfloat16>(kn);
    p.pos = ptr<const int32_t>(pos);
    p.batch = ptr<const int32_t>(batch);
    if (slots)
        check(slots->is_cuda() && slots->is_contiguous() && slots->scalar_type() == at::kInt &&
                  slots->numel() == pos.numel(),
              "qk_norm_rope_kv slots: int32 [T]");
    p.slot = optr<const int32_t>(slots);
    p.q = ptr<__nv_bfloat16>(q);
    p.kc = ptr<__nv_bfloat16>(kc);
    p.vc = ptr<__nv_bfloat16>(vc);
    p.Hq = int(hq);
    p.Hkv = int(hkv);
    p.D = int(kc.size(-1));
    p.L = int(kc.size(-2));
    p.T = int(pos.numel());
    p.theta = float(theta);
    p.eps = float(eps);
    check(qkv.size(-1) == (hq + 2 * hkv) * p.D, "qkv width");
    c10::cuda::CUDAGuard g(qkv.device());
    check_rc(xt_qk_norm_rope_kv(&p, stream()), "qk_norm_rope_kv");
}

void attn_decode(const Tensor &q, const Tensor &kc, const Tensor &vc, const Tensor &seqlens, const Tensor &out,
                 const Tensor &ws_o, const Tensor &ws_ml, const Tensor &counters, int64_t splits, double scale) {
    cuda_contig(q, "q");
    cuda_contig(kc, "k_cache");
    AttnDecodeParams p{};
    p.q = ptr<const __nv_bfloat16>(q);
    p.kc = ptr<const __nv_bfloat16>(kc);
    p.vc = ptr<const __nv_bfloat16>(vc);
    p.seqlens = ptr<const int32_t>(seqlens);
    p.out = ptr<__nv_bfloat16>(out);
    p.ws_o = ptr<float>(ws_o);
    p.ws_ml = ptr<float>(ws_ml);
    p.counters = ptr<uint32_t>(counters);
    const int B = int(q.size(0));
    p.Hq = int(q.size(1));
    p.Hkv = int(kc.size(1));
    p.L = int(kc.size(2));
    p.splits = int(splits);
    p.scale_log2 = float(scale * 1.4426950408889634);
    const int G = p.Hq / p.Hkv;
    check(ws_o.numel() >= int64_t(B) * p.Hkv * splits * G * 128, "ws_o too small");
    check(ws_ml.numel() >= int64_t(B) * p.Hkv * splits * G * 2, "ws_ml too small");
    check(counters.numel() >= int64_t(B) * p.Hkv, "counters too small");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_attn_decode(&p, B, stream()), "attn_decode");
}

void moe_route(const Tensor &x, const Tensor &wr, const std::optional<Tensor> &bias, const std::optional<Tensor> &corr,
               const std::optional<Tensor> &table, const std::optional<Tensor> &shared_slots, const Tensor &ids,
               const Tensor &w, const Tensor &slots, const Tensor &ws_logits, const Tensor &ws_count, int64_t k,
               int64_t mode, int64_t n_group, int64_t topk_group, bool renorm, double scale, int64_t layer,
               int64_t mailbox, const std::optional<Tensor> &active, const std::optional<Tensor> &logits_in,
               const std::optional<Tensor> &cold_index, int64_t share_min, int64_t host_base,
               const std::optional<Tensor> &claim, const std::optional<Tensor> &claim_list,
               const std::optional<Tensor> &claim_count, int64_t stage_max, int64_t stage_slot0) {
    cuda_contig(x, "x");
    cuda_contig(wr, "router weight");
    RouteParams p{};
    p.x = ptr<const __nv_bfloat16>(x);
    p.wr = ptr<const __nv_bfloat16>(wr);
    p.bias = optr<const float>(bias);
    p.corr = optr<const float>(corr);
    p.table = optr<const int32_t>(table);
    p.shared_slots = optr<const int32_t>(shared_slots);
    p.active = optr<const int32_t>(active);
    p.logits_in = optr<const float>(logits_in);
    p.cold_index = optr<const int32_t>(cold_index);
    p.share_min = int(share_min);
    p.host_base = int(host_base);
    if (cold_index)
        check(cold_index->scalar_type() == at::kInt && cold_index->numel() >= wr.size(0) &&
                  (host_base > 0 || share_min == 0),
              "cold_index: int32 [E] and a positive host_base");
    p.stage_max = int(stage_max);
    if (stage_max > 0) {
        check(cold_index && claim && claim_list && claim_count && !logits_in, "PCIe staging: cold_index and claims");
        check(claim->scalar_type() == at::kInt && claim->numel() >= wr.size(0) && claim_list->numel() >= wr.size(0) &&
                  claim_count->numel() >= 1,
              "PCIe staging: claim and claim_list int32 [E], claim_count [1]");
        p.claim = ptr<int32_t>(*claim);
        p.claim_list = ptr<int32_t>(*claim_list);
        p.claim_count = ptr<int32_t>(*claim_count);
        p.stage_slot0 = int(stage_slot0);
    }
    if (logits_in)
        check(logits_in->scalar_type() == at::kFloat && logits_in->numel() >= x.size(0) * wr.size(0) && mailbox == 0,
              "logits_in: fp32 [m, E], no mailbox");
    if (active) check(active->numel() >= x.size(0) && active->scalar_type() == at::kInt, "active: int32 [m] flags");
    p.ids = ptr<int32_t>(ids);
    p.w = ptr<float>(w);
    p.slots = ptr<int32_t>(slots);
    p.ws_logits = ptr<float>(ws_logits);
    p.ws_count = ptr<uint32_t>(ws_count);
    p.m = int(x.size(0));
    p.H = int(x.size(1));
    p.E = int(wr.size(0));
    p.k = int(k);
    p.n_shared = shared_slots.has_value() ? int(shared_slots->numel()) : 0;
    p.mode = int(mode);
    p.n_group = int(n_group);
    p.topk_group = int(topk_group);
    p.renorm = renorm;
    p.scale = float(scale);
    p.layer = int(layer);
    check(ids.numel() >= int64_t(p.m) * (p.k + p.n_shared), "ids too small");
    check(p.k <= p.E, "k > experts");
    check(ws_logits.numel() >= int64_t(p.m) * p.E && ws_count.numel() >= p.m, "router scratch too small");
    XtMailbox mb = mailbox_view(mailbox);
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_moe_route(&p, &mb, mailbox != 0, stream()), "moe_route");
}

void moe_gate_up(const Tensor &x, const Tensor &slots, const Tensor &w13, const Tensor &s13, const Tensor &g13,
                 const Tensor &mid, int64_t fmt, double limit, double alpha, double beta,
                 const std::optional<Tensor> &peer, int64_t spr, const std::optional<Tensor> &host,
                 int64_t host_base) {
    cuda_contig(w13, "w13");
    cuda_contig(s13, "s13");
    GateUpParams p{};
    p.x = ptr<const __nv_bfloat16>(x);
    p.slots = ptr<const int32_t>(slots);
    p.w13 = ptr<const uint8_t>(w13);
    p.s13 = ptr<const uint8_t>(s13);
    p.g13 = ptr<const float>(g13);
    check(mid.scalar_type() == at::kHalf, "moe_gate_up: mid must be float16");
    p.mid = ptr<__half>(mid);
    p.routes = int(slots.numel());
    p.kk = int(slots.size(-1));
    p.H = int(x.size(-1));
    p.I = int(w13.size(1) / 2);
    p.fmt = int(fmt);
    p.limit = float(limit);
    p.alpha = float(alpha);
    p.beta = float(beta);
    p.peer = peer ? reinterpret_cast<const unsigned long long *>(peer->data_ptr<int64_t>()) : nullptr;
    p.spr = int(spr);
    if (peer) check(peer->is_cuda() && peer->scalar_type() == at::kLong && peer->numel() % 6 == 0 && spr > 0,
                    "peer: int64 [W * 6] device table and slots per rank");
    p.host = host ? reinterpret_cast<const unsigned long long *>(host->data_ptr<int64_t>()) : nullptr;
    p.host_base = int(host_base);
    if (host) check(host->is_cuda() && host->scalar_type() == at::kLong && host->numel() == 6 && host_base > 0,
                    "host: int64 [6] device table of the pinned host pool and a positive host_base");
    check(mid.numel() >= int64_t(p.routes) * p.I, "mid too small");
    check(w13.size(2) * 2 == p.H, "w13 / x hidden mismatch");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_moe_gate_up(&p, stream()), "moe_gate_up");
}

void moe_down(const Tensor &mid, const Tensor &slots, const Tensor &w, const Tensor &w2, const Tensor &s2,
              const Tensor &g2, const std::optional<Tensor> &add, const Tensor &out,
              const std::optional<Tensor> &out_f32, const std::optional<Tensor> &gpu_part, int64_t fmt,
              int64_t mailbox, const std::optional<Tensor> &peer, int64_t spr, const std::optional<Tensor> &host,
              int64_t host_base) {
    cuda_contig(w2, "w2");
    DownParams p{};
    p.peer = peer ? reinterpret_cast<const unsigned long long *>(peer->data_ptr<int64_t>()) : nullptr;
    p.spr = int(spr);
    p.host = host ? reinterpret_cast<const unsigned long long *>(host->data_ptr<int64_t>()) : nullptr;
    p.host_base = int(host_base);
    if (host) check(host->is_cuda() && host->scalar_type() == at::kLong && host->numel() == 6 && host_base > 0,
                    "host: int64 [6] device table of the pinned host pool and a positive host_base");
    if (peer) check(peer->is_cuda() && peer->scalar_type() == at::kLong && peer->numel() % 6 == 0 && spr > 0,
                    "peer: int64 [W * 6] device table and slots per rank");
    check(mid.scalar_type() == at::kHalf, "moe_down: mid must be float16");
    p.mid = ptr<const __half>(mid);
    p.slots = ptr<const int32_t>(slots);
    p.w = ptr<const float>(w);
    p.w2 = ptr<const uint8_t>(w2);
    p.s2 = ptr<const uint8_t>(s2);
    p.g2 = ptr<const float>(g2);
    p.add = optr<const __nv_bfloat16>(add);
    p.out = ptr<__nv_bfloat16>(out);
    p.out_f32 = optr<float>(out_f32);
    p.gpu_part = optr<float>(gpu_part);
    p.kk = int(slots.size(-1));
    p.H = int(w2.size(1));
    p.I = int(w2.size(2) * 2);
    p.fmt = int(fmt);
    const int m = int(slots.size(0));
    check(p.H % 4 == 0, "hidden % 4");
    XtMailbox mb = mailbox_view(mailbox);
    c10::cuda::CUDAGuard g(out.device());
    check_rc(xt_moe_down(&p, &mb, mailbox != 0, m, stream()), "moe_down");
}

void gemv(const Tensor &x, const Tensor &w, const std::optional<Tensor> &add, const Tensor &out) {
    cuda_contig(x, "x");
    cuda_contig(w, "w");
    cuda_contig(out, "out");
    check(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemv wants bf16");
    const int K = int(x.size(-1)), m = int(x.numel() / K), N = int(w.size(0));
    check(w.size(1) == K && out.numel() == int64_t(m) * N, "gemv shapes");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_gemv_bf16(x.data_ptr(), w.data_ptr(), optr<void>(add), out.data_ptr(), m, N, K, stream()), "gemv");
}

void fp8_rows(const Tensor &tab, const Tensor &scales, const std::optional<Tensor> &ids, int64_t lo, int64_t hi,
              int64_t blk, const Tensor &out) {
    cuda_contig(tab, "tab");
    cuda_contig(scales, "scales");
    cuda_contig(out, "out");
    check(tab.scalar_type() == at::kByte && scales.scalar_type() == at::kByte && out.scalar_type() == at::kBFloat16,
          "fp8_rows: uint8 payload and scales, bf16 out");
    const int64_t dim = tab.size(-1);
    const int64_t n = ids ? ids->numel() : tab.numel() / dim;
    check(out.numel() == n * dim && scales.size(-1) == dim / blk, "fp8_rows shapes");
    if (ids) check(ids->is_cuda() && ids->is_contiguous() && ids->scalar_type() == at::kLong, "fp8_rows: int64 ids");
    c10::cuda::CUDAGuard g(tab.device());
    check_rc(xt_fp8_rows(tab.data_ptr(), scales.data_ptr(), ids ? ids->data_ptr<int64_t>() : nullptr, lo, hi, int(n),
                         int(dim), int(blk), out.data_ptr(), stream()),
             "fp8_rows");
}

void gemv_fp8(const Tensor &x, const Tensor &w, const Tensor &s, const std::optional<Tensor> &add, const Tensor &out) {
    cuda_contig(x, "x");
    cuda_contig(w, "w");
    cuda_contig(s, "s");
    cuda_contig(out, "out");
    check(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kByte && s.scalar_type() == at::kFloat,
          "gemv_fp8: bf16 x, uint8 (E4M3) w, fp32 scales");
    const int K = int(x.size(-1)), m = int(x.numel() / K), N = int(w.size(0));
    check(w.size(1) == K && s.size(0) == N && s.size(1) == K / 128 && out.numel() == int64_t(m) * N, "gemv_fp8 shapes");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_gemv_fp8(x.data_ptr(), w.data_ptr(), s.data_ptr<float>(), optr<void>(add), out.data_ptr(), m, N, K,
                         stream()),
             "gemv_fp8");
}

void spec_truncate(const Tensor &q, const Tensor &tokens, const std::optional<Tensor> &topk, const Tensor &flags,
                   double threshold) {
    check(q.is_cuda() && q.dim() == 3 && q.scalar_type() == at::kFloat && q.stride(2) == 1, "spec_truncate: fp32 q [B, S, V]");
    const int64_t B = q.size(0), S = q.size(1), V = q.size(2);
    cuda_contig(tokens, "tokens");
    cuda_contig(flags, "flags");
    check(tokens.scalar_type() == at::kLong && tokens.numel() == B * (S + 1), "spec_truncate: int64 tokens [B, S + 1]");
    check(flags.scalar_type() == at::kInt && flags.numel() >= B * (S + 1), "spec_truncate: int32 flags [B * (S + 1)]");
    if (topk) check(topk->is_cuda() && topk->scalar_type() == at::kInt && topk->numel() >= B, "spec_truncate: int32 top_k");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_spec_truncate(q.data_ptr<float>(), tokens.data_ptr<int64_t>(), topk ? topk->data_ptr<int32_t>() : nullptr,
                              flags.data_ptr<int32_t>(), float(threshold), q.stride(0), q.stride(1), int(B), int(S),
                              int(V), stream()),
             "spec_truncate");
}

void gather_rows(const Tensor &x, const Tensor &src, const Tensor &X) {
    cuda_contig(x, "x");
    cuda_contig(src, "src");
    cuda_contig(X, "X");
    const int H = int(x.size(-1));
    check(x.scalar_type() == at::kBFloat16 && X.scalar_type() == at::kBFloat16 && src.scalar_type() == at::kInt &&
              X.numel() == src.numel() * H,
          "gather_rows shapes");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_gather_rows(x.data_ptr(), src.data_ptr<int32_t>(), X.data_ptr(), int(src.numel()), H, stream()),
             "gather_rows");
}

void route_combine(const Tensor &Ya, const Tensor &da, const std::optional<Tensor> &Yb,
                   const std::optional<Tensor> &db, const std::optional<Tensor> &add, const Tensor &out) {
    cuda_contig(Ya, "Ya");
    cuda_contig(da, "da");
    cuda_contig(out, "out");
    const int H = int(out.size(-1)), m = int(out.numel() / H);
    check(Ya.scalar_type() == at::kFloat && da.scalar_type() == at::kInt && da.numel() % m == 0, "route_combine a");
    if (Yb) check(db && Yb->scalar_type() == at::kFloat && db->scalar_type() == at::kInt && db->numel() % m == 0,
                  "route_combine b");
    check(out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16, "route_combine out dtype");
    if (add) check(add->scalar_type() == at::kBFloat16 && add->numel() == out.numel(), "route_combine add");
    c10::cuda::CUDAGuard g(out.device());
    check_rc(xt_route_combine(Ya.data_ptr<float>(), da.data_ptr<int32_t>(), int(da.numel() / m),
                              Yb ? Yb->data_ptr<float>() : nullptr, db ? db->data_ptr<int32_t>() : nullptr,
                              db ? int(db->numel() / m) : 0, add ? add->data_ptr() : nullptr, out.data_ptr(),
                              out.scalar_type() == at::kFloat, m, H, stream()),
             "route_combine");
}

void gemm_tc_f32(const Tensor &a, const Tensor &b, const Tensor &out, const Tensor &err) {
    cuda_contig(a, "a");
    cuda_contig(b, "b");
    cuda_contig(out, "out");
    check(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kFloat,
          "gemm_tc_f32: bf16 operands, fp32 out");
    const int K = int(a.size(-1)), M = int(a.numel() / K), N = int(b.size(0));
    check(b.size(1) == K && out.numel() == int64_t(M) * N, "gemm_tc_f32 shapes");
    c10::cuda::CUDAGuard g(a.device());
    check_rc(xt_gemm_tc_f32(a.data_ptr(), b.data_ptr(), out.data_ptr<float>(), M, N, K, err.data_ptr<int>(), stream()),
             "gemm_tc_f32");
}

void fp8_dequant(const Tensor &w, const Tensor &s, const Tensor &out) {
    cuda_contig(w, "w");
    cuda_contig(s, "s");
    cuda_contig(out, "out");
    const int N = int(w.size(0)), K = int(w.size(1));
    check(w.scalar_type() == at::kByte && s.scalar_type() == at::kFloat && out.scalar_type() == at::kBFloat16 &&
              s.size(0) == N && s.size(1) == K / 128 && out.numel() == int64_t(N) * K,
          "fp8_dequant shapes");
    c10::cuda::CUDAGuard g(w.device());
    check_rc(xt_fp8_dequant(w.data_ptr(), s.data_ptr<float>(), out.data_ptr(), N, K, stream()), "fp8_dequant");
}

void gemm_tc(const Tensor &a, const Tensor &b, const std::optional<Tensor> &residual, const Tensor &out,
             const Tensor &err) {
    cuda_contig(a, "a");
    cuda_contig(b, "b");
    cuda_contig(out, "out");
    check(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_tc wants bf16");
    const int K = int(a.size(-1)), M = int(a.numel() / K), N = int(b.size(0));
    check(b.size(1) == K && out.numel() == int64_t(M) * N, "gemm_tc shapes");
    check(err.scalar_type() == at::kInt && err.is_cuda(), "gemm_tc error word: int32 CUDA tensor");
    c10::cuda::CUDAGuard g(a.device());
    check_rc(xt_gemm_tc(a.data_ptr(), b.data_ptr(), out.data_ptr(), optr<void>(residual), M, N, K, ptr<int>(err),
                        stream()),
             "gemm_tc");
}

void ep_moe(const Tensor &x, const Tensor &ids, const Tensor &w, const Tensor &peer, const Tensor &state,
            const Tensor &mid, const Tensor &w13, const Tensor &s13, const Tensor &g13, const Tensor &w2,
            const Tensor &s2, const Tensor &g2, const std::optional<Tensor> &add, const Tensor &out, const Tensor &err,
            int64_t W, int64_t rank, int64_t E, int64_t fmt, int64_t R, std::vector<int64_t> offsets, double timeout_s,
            int64_t phases, const std::optional<Tensor> &slots, int64_t spr, int64_t mailbox,
            const std::optional<Tensor> &st_w13, const std::optional<Tensor> &st_s13,
            const std::optional<Tensor> &st_w2, const std::optional<Tensor> &st_s2,
            const std::optional<Tensor> &st_g13, const std::optional<Tensor> &st_g2, int64_t stage_base) {
    cuda_contig(x, "x");
    xt::EpParams p{};
    p.W = int(W);
    p.rank = int(rank);
    p.E = int(E);
    p.El = slots.has_value() && slots->defined() ? int(spr) : int(E / W);
    p.slots = optr<const int32_t>(slots);
    if (p.slots) check(spr > 0 && slots->scalar_type() == at::kInt && slots->is_contiguous(), "ep slots");
    p.mb = mailbox_view(mailbox);
    p.use_mb = mailbox ? 1 : 0;
    static const int by_expert = [] {   // XTIER_EP_ORDER=0: the expert streams take the routes in arrival order
        const char *v = getenv("XTIER_EP_ORDER");
        return v && *v == '0' ? 0 : 1;
    }();
    p.by_expert = by_expert;
    p.H = int(x.size(1));
    p.I = int(w13.size(1) / 2);
    p.k = int(ids.size(1));
    p.T = int(x.size(0));
    p.R = int(R);
    p.fmt = int(fmt);
    p.peer = ptr<const uint64_t>(peer);
    check(offsets.size() == 6, "ep offsets");
    p.off_rx = size_t(offsets[0]);
    p.off_meta = size_t(offsets[1]);
    p.off_cnt = size_t(offsets[2]);
    p.off_flag = size_t(offsets[3]);
    p.off_ret = size_t(offsets[4]);
    p.off_rflag = size_t(offsets[5]);
    p.x = ptr<const __nv_bfloat16>(x);
    p.ids = ptr<const int32_t>(ids);
    p.w = ptr<const float>(w);
    p.state = ptr<uint32_t>(state);
    check(mid.scalar_type() == at::kHalf, "ep mid scratch must be float16");
    p.mid = ptr<__half>(mid);
    p.w13 = ptr<const uint8_t>(w13);
    p.s13 = ptr<const uint8_t>(s13);
    p.g13 = ptr<const float>(g13);
    p.w2 = ptr<const uint8_t>(w2);
    p.s2 = ptr<const uint8_t>(s2);
    p.g2 = ptr<const float>(g2);
    p.add = optr<const __nv_bfloat16>(add);
    p.out = ptr<__nv_bfloat16>(out);
    p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
    p.error = ptr<int>(err);
    if (stage_base > 0) {
        check(st_w13 && st_s13 && st_w2 && st_s2 && st_g13 && st_g2 && p.slots, "ep: staging pools");
        check(st_g13->scalar_type() == at::kFloat && st_g2->scalar_type() == at::kFloat, "ep: staging scales fp32");
        p.st_w13 = ptr<const uint8_t>(*st_w13);
        p.st_s13 = ptr<const uint8_t>(*st_s13);
        p.st_w2 = ptr<const uint8_t>(*st_w2);
        p.st_s2 = ptr<const uint8_t>(*st_s2);
        p.st_g13 = ptr<const float>(*st_g13);
        p.st_g2 = ptr<const float>(*st_g2);
        p.stage_base = int(stage_base);
    }
    check(p.T * p.k <= p.R, "ep: more routes than a receive region holds");
    check(mid.numel() >= int64_t(W) * R * p.I, "ep mid scratch too small");
    c10::cuda::CUDAGuard g(x.device());
    for (int ph = 0; ph < 4; ++ph)
        if ((phases >> ph) & 1) check_rc(xt_ep_moe(&p, ph, stream()), "ep_moe");
}

void ep_stage(const Tensor &claim_list, const Tensor &claim, const Tensor &claim_count, const Tensor &done,
              const Tensor &cold_index, std::vector<int64_t> bases, int64_t stride, std::vector<int64_t> piece_off,
              std::vector<int64_t> piece_bytes, const Tensor &w13, const Tensor &s13, const Tensor &w2,
              const Tensor &s2, const Tensor &g13, const Tensor &g2, const Tensor &src_g13, const Tensor &src_g2,
              int64_t I, int64_t H, int64_t fmt, int64_t chunks) {
    xt::StageParams p{};
    check(bases.size() >= 1 && bases.size() <= 8 && piece_off.size() == 6 && piece_bytes.size() == 6,
          "ep_stage: 1-8 node bases and 6 pieces");
    const int E = int(claim.numel());
    check(claim.scalar_type() == at::kInt && claim_list.numel() >= E && cold_index.numel() >= E &&
              claim_count.numel() >= 1 && done.numel() >= 1,
          "ep_stage: claim tensors");
    check(src_g13.scalar_type() == at::kFloat && src_g2.scalar_type() == at::kFloat && g13.scalar_type() == at::kFloat &&
              g2.scalar_type() == at::kFloat,
          "ep_stage: global scales fp32");
    p.claim_list = ptr<const int32_t>(claim_list);
    p.claim = ptr<int32_t>(claim);
    p.claim_count = ptr<int32_t>(claim_count);
    p.done = ptr<uint32_t>(done);
    p.cold_index = ptr<const int32_t>(cold_index);
    p.nodes = int(bases.size());
    for (size_t n = 0; n < bases.size(); ++n) p.base[n] = static_cast<unsigned long long>(bases[n]);
    p.stride = static_cast<unsigned long long>(stride);
    for (int q = 0; q < 6; ++q) {
        p.piece_off[q] = static_cast<unsigned long long>(piece_off[q]);
        p.piece_bytes[q] = static_cast<unsigned long long>(piece_bytes[q]);
    }
    p.w13 = ptr<uint8_t>(w13);
    p.s13 = ptr<uint8_t>(s13);
    p.w2 = ptr<uint8_t>(w2);
    p.s2 = ptr<uint8_t>(s2);
    p.g13 = ptr<float>(g13);
    p.g2 = ptr<float>(g2);
    p.src_g13 = ptr<const float>(src_g13);
    p.src_g2 = ptr<const float>(src_g2);
    p.stage_max = int(w13.size(0));
    p.E = E;
    p.I = int(I);
    p.H = int(H);
    p.bs = fmt == 0 ? 16 : 32;
    p.chunks = int(chunks);
    const int64_t I_ = I, H_ = H, N = p.nodes;
    const int64_t want[6] = {I_ / N * (H_ / 2), I_ / N * (H_ / 2), I_ / N * (H_ / p.bs), I_ / N * (H_ / p.bs),
                             H_ / N * (I_ / 2), H_ / N * (I_ / p.bs)};
    for (int q = 0; q < 6; ++q) check(piece_bytes[q] == want[q], "ep_stage: engine piece sizes differ from the pool");
    check(w13.numel() == int64_t(p.stage_max) * 2 * I * (H / 2) && s13.numel() == int64_t(p.stage_max) * 2 * I * (H / p.bs) &&
              w2.numel() == int64_t(p.stage_max) * H * (I / 2) && s2.numel() == int64_t(p.stage_max) * H * (I / p.bs),
          "ep_stage: staging pool shapes");
    c10::cuda::CUDAGuard g(w13.device());
    check_rc(xt_ep_stage(&p, stream()), "ep_stage");
}

void qsa_kv_write(const Tensor &x, const Tensor &slots, const Tensor &codes, const Tensor &scales) {
    cuda_contig(x, "qsa kv rows");
    check(x.dim() == 3 && x.scalar_type() == at::kBFloat16, "qsa kv rows: bf16 [T, Hkv, D]");
    const int T = int(x.size(0)), H = int(x.size(1)), D = int(x.size(2));
    check(slots.scalar_type() == at::kLong && slots.numel() == T && slots.is_contiguous(), "qsa slots: int64 [T]");
    check(codes.dim() == 3 && codes.size(1) == H && codes.size(2) == D / 2 && scales.dim() == 3 &&
              scales.size(1) == H && scales.size(2) == D / 16 && codes.size(0) == scales.size(0),
          "qsa cache: codes [slots, Hkv, D/2], scales [slots, Hkv, D/16]");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_qsa_kv_write(x.data_ptr(), ptr<const int64_t>(slots), T, H, D, codes.data_ptr(), scales.data_ptr(),
                             stream()),
             "qsa_kv_write");
}

void qsa_decode(const Tensor &q, const Tensor &idx, const Tensor &kc, const Tensor &ks, const Tensor &vc,
                const Tensor &vs, const Tensor &part_o, const Tensor &part_ml, const Tensor &out, double scale) {
    cuda_contig(q, "qsa q");
    check(q.dim() == 3 && q.scalar_type() == at::kBFloat16, "qsa q: bf16 [B, Hq, D]");
    const int B = int(q.size(0)), Hq = int(q.size(1)), D = int(q.size(2)), Hkv = int(kc.size(1));
    check(idx.scalar_type() == at::kInt && idx.dim() == 2 && idx.size(0) == B && idx.is_contiguous(),
          "qsa idx: int32 [B, nsel]");
    const int nsel = int(idx.size(1));
    check(Hkv > 0 && Hq % Hkv == 0 && kc.size(2) == D / 2 && vc.sizes() == kc.sizes() && vs.sizes() == ks.sizes(),
          "qsa cache shapes");
    const int64_t splits = (nsel + 31) / 32;
    check(part_o.numel() >= int64_t(B) * Hq * splits * D && part_ml.numel() >= int64_t(B) * Hq * splits * 2,
          "qsa scratch too small");
    check(out.numel() == q.numel() && out.scalar_type() == at::kBFloat16, "qsa out: bf16 like q");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_qsa_decode(q.data_ptr(), ptr<const int32_t>(idx), B, nsel, Hq, Hkv, D, kc.data_ptr(), ks.data_ptr(),
                           vc.data_ptr(), vs.data_ptr(), ptr<float>(part_o), ptr<float>(part_ml), out.data_ptr(),
                           float(scale), stream()),
             "qsa_decode");
}

xt::TpParams tp_params(const Tensor &peer, const Tensor &state, const Tensor &out, const Tensor &err, int64_t M,
                       int64_t N, int64_t K, int64_t W, int64_t rank, const std::vector<int64_t> &offs,
                       double timeout_s) {
    check(offs.size() == 4, "tp offsets: data0, data1, flags0, flags1");
    xt::TpParams p{};
    p.M = int(M);
    p.N = int(N);
    p.K = int(K);
    p.W = int(W);
    p.rank = int(rank);
    p.peer = ptr<const uint64_t>(peer);
    p.off_data[0] = size_t(offs[0]);
    p.off_data[1] = size_t(offs[1]);
    p.off_flags[0] = size_t(offs[2]);
    p.off_flags[1] = size_t(offs[3]);
    p.state = ptr<uint32_t>(state);
    p.out = ptr<__nv_bfloat16>(out);
    p.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
    p.error = ptr<int>(err);
    return p;
}

void gemm_rs(const Tensor &a, const Tensor &b, const Tensor &peer, const Tensor &state,
             const std::optional<Tensor> &residual, const Tensor &out, const Tensor &err, int64_t W, int64_t rank,
             std::vector<int64_t> offs, double timeout_s) {
    cuda_contig(a, "a");
    cuda_contig(b, "b");
    cuda_contig(out, "out");
    const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
    check(b.size(1) == K && out.numel() == M / W * N, "gemm_rs shapes");
    xt::TpParams p = tp_params(peer, state, out, err, M, N, K, W, rank, offs, timeout_s);
    p.residual = optr<const __nv_bfloat16>(residual);
    c10::cuda::CUDAGuard g(a.device());
    check_rc(xt_gemm_rs(a.data_ptr(), b.data_ptr(), &p, stream()), "gemm_rs");
}

void ag_gemm(const Tensor &a_shard, const Tensor &b, const Tensor &peer, int64_t local_base, const Tensor &state,
             const Tensor &out, const Tensor &err, int64_t W, int64_t rank, std::vector<int64_t> offs,
             double timeout_s) {
    cuda_contig(a_shard, "a_shard");
    cuda_contig(b, "b");
    cuda_contig(out, "out");
    const int64_t M = a_shard.size(0) * W, K = a_shard.size(1), N = b.size(0);
    check(b.size(1) == K && out.numel() == M * N, "ag_gemm shapes");
    xt::TpParams p = tp_params(peer, state, out, err, M, N, K, W, rank, offs, timeout_s);
    p.a_shard = ptr<const __nv_bfloat16>(a_shard);
    c10::cuda::CUDAGuard g(a_shard.device());
    check_rc(xt_ag_gemm(b.data_ptr(), reinterpret_cast<const void *>(local_base), &p, stream()), "ag_gemm");
}

void l2_prefetch(const Tensor &ptrs, const Tensor &bytes, int64_t ctas) {
    check(ptrs.scalar_type() == at::kLong && bytes.scalar_type() == at::kLong && ptrs.numel() == bytes.numel(),
          "l2_prefetch: int64 pointer and size tensors of one length");
    c10::cuda::CUDAGuard g(ptrs.device());
    check_rc(xt_l2_prefetch(ptr<const uint64_t>(ptrs), ptr<const uint64_t>(bytes), int(ptrs.numel()), int(ctas),
                            stream()),
             "l2_prefetch");
}

void mla_kv_write(const Tensor &lat, const Tensor &slot, const Tensor &codes, const Tensor &scales, const Tensor &rope) {
    cuda_contig(lat, "lat");
    check(lat.size(-1) == 576 && slot.scalar_type() == at::kLong && slot.numel() == lat.size(0), "mla_kv_write shapes");
    check(codes.size(-1) == 256 && scales.size(-1) == 32 && rope.size(-1) == 64, "mla cache layout");
    c10::cuda::CUDAGuard g(lat.device());
    check_rc(xt_mla_kv_write(lat.data_ptr(), ptr<const int64_t>(slot), codes.data_ptr(), scales.data_ptr(),
                             rope.data_ptr(), int(lat.size(0)), stream()),
             "mla_kv_write");
}

void mla_decode(const Tensor &q, const Tensor &idx, const Tensor &codes, const Tensor &scales, const Tensor &rope,
                const Tensor &kg, const Tensor &vt, const Tensor &part_o, const Tensor &part_ml, const Tensor &out,
                double scale, const Tensor &err) {
    cuda_contig(q, "q");
    cuda_contig(idx, "idx");
    const int64_t Q = q.size(0), nsel = idx.size(1);
    check(q.size(1) == 128 && q.size(2) == 576 && idx.size(0) == Q && idx.scalar_type() == at::kInt, "mla_decode q/idx");
    check(kg.numel() >= Q * nsel * 576 && vt.numel() >= Q * 512 * nsel, "mla_decode gather scratch too small");
    check(part_o.numel() >= Q * (nsel / 128) * 128 * 512 && part_ml.numel() >= Q * (nsel / 128) * 128 * 2,
          "mla_decode partial scratch too small");
    check(out.numel() == Q * 128 * 512, "mla_decode out [Q, 128, 512]");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_mla_decode(q.data_ptr(), ptr<const int32_t>(idx), int(Q), int(nsel), codes.data_ptr(),
                           scales.data_ptr(), rope.data_ptr(), kg.data_ptr(), vt.data_ptr(), ptr<float>(part_o),
                           ptr<float>(part_ml), out.data_ptr(), float(scale), ptr<int>(err), stream()),
             "mla_decode");
}

// q [Q, 128, 576] (latent then rotary values), or with q_rope: q [Q, 128, 512] and q_rope [Q, 128, 64]; q, q_rope and
// out [Q, 128, 512] may be strided views (unit stride along the last dim).
void mla_flash(const Tensor &q, const Tensor &idx, const Tensor &codes, const Tensor &scales, const Tensor &rope,
               const std::optional<Tensor> &part_o, const std::optional<Tensor> &part_ml, const Tensor &out,
               double scale, int64_t splits, const Tensor &err, const std::optional<Tensor> &q_rope) {
    cuda_contig(idx, "idx");
    auto rows_ok = [](const Tensor &t, int64_t d) {
        return t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.size(1) == 128 && t.size(2) == d &&
               t.stride(2) == 1;
    };
    const int64_t Q = q.size(0), nsel = idx.size(1);
    check(rows_ok(q, q_rope ? 512 : 576) && (!q_rope || (rows_ok(*q_rope, 64) && q_rope->size(0) == Q)),
          "mla_flash: q [Q, 128, 576] bf16, or q [Q, 128, 512] and q_rope [Q, 128, 64] (unit stride along the last dim)");
    check(idx.size(0) == Q && idx.scalar_type() == at::kInt && nsel % 64 == 0,
          "mla_flash idx [Q, nsel] int32 (nsel % 64 == 0)");
    check(rows_ok(out, 512) && out.size(0) == Q, "mla_flash out [Q, 128, 512] bf16 (unit stride along the last dim)");
    const int64_t nblk = nsel / 64, bps = (nblk + splits - 1) / splits, eff = (nblk + bps - 1) / bps;
    if (eff > 1)
        check(part_o && part_ml && part_o->numel() >= Q * eff * 128 * 512 && part_ml->numel() >= Q * eff * 128 * 2 &&
                  out.is_contiguous(),
              "mla_flash: split partials too small, or a strided out with splits");
    const auto *qp = static_cast<const __nv_bfloat16 *>(q.data_ptr());
    const void *qr = q_rope ? q_rope->data_ptr() : static_cast<const void *>(qp + 512);
    const int64_t qr_ts = q_rope ? q_rope->stride(0) : q.stride(0), qr_hs = q_rope ? q_rope->stride(1) : q.stride(1);
    static const bool bounds = [] {   // XTIER_DEBUG_BOUNDS: selected slots checked against the cache size
        const char *v = getenv("XTIER_DEBUG_BOUNDS");
        return v && *v && *v != '0';
    }();
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_mla_flash(qp, q.stride(0), q.stride(1), qr, qr_ts, qr_hs, ptr<const int32_t>(idx), int(Q), int(nsel),
                          codes.data_ptr(), scales.data_ptr(), rope.data_ptr(), optr<float>(part_o),
                          optr<float>(part_ml), out.data_ptr(), out.stride(0), out.stride(1), float(scale),
                          int(splits), bounds ? int(codes.size(0)) : 0, ptr<int>(err), stream()),
             "mla_flash");
}

// Causal GQA prefill attention of q [T, Hq, 128] (a view with unit stride along the last dim) at positions
// start .. start + T - 1 over row `row` of the caches k, v [B, Hkv, max_len, 128] (contiguous BF16); out [T, Hq, 128]
// likewise a view.
void attn_prefill(const Tensor &q, const Tensor &k, const Tensor &v, const Tensor &out, int64_t row, int64_t start,
                  double scale, const Tensor &err, const std::optional<Tensor> &tree_mask) {
    auto view_ok = [](const Tensor &t) {
        return t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.size(2) == 128 && t.stride(2) == 1;
    };
    check(view_ok(q) && view_ok(out) && out.size(0) == q.size(0) && out.size(1) == q.size(1),
          "attn_prefill: q and out [T, Hq, 128] bf16 (unit stride along the last dim)");
    cuda_contig(k, "k");
    cuda_contig(v, "v");
    check(k.dim() == 4 && k.size(3) == 128 && k.sizes() == v.sizes() && k.scalar_type() == at::kBFloat16 &&
              v.scalar_type() == at::kBFloat16,
          "attn_prefill: k, v [B, Hkv, max_len, 128] bf16");
    const int64_t T = q.size(0), Hq = q.size(1), Hkv = k.size(1), L = k.size(2);
    check(row >= 0 && row < k.size(0) && start >= 0 && start + T <= L && Hq % Hkv == 0,
          "attn_prefill: row / start out of range, or Hq not a multiple of Hkv");
    check(err.is_cuda() && err.scalar_type() == at::kInt, "attn_prefill err int32");
    if (tree_mask)
        check(tree_mask->is_cuda() && tree_mask->is_contiguous() && tree_mask->scalar_type() == at::kLong &&
                  tree_mask->numel() == T && T <= 64,
              "attn_prefill tree_mask: int64 [T], T <= 64");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_attn_prefill(q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.size(0) * Hkv * L,
                             row * Hkv * L, L, int(T), int(start), int(Hq), int(Hkv), out.data_ptr(), out.stride(0),
                             out.stride(1), float(scale),
                             tree_mask ? static_cast<const unsigned long long *>(tree_mask->data_ptr()) : nullptr,
                             ptr<int>(err), stream()),
             "attn_prefill");
}

void dsa_key_write(const Tensor &k, const Tensor &slot, const Tensor &codes, const Tensor &kscale) {
    cuda_contig(k, "k");
    check(k.size(-1) == 128 && slot.scalar_type() == at::kLong && slot.numel() == k.size(0) &&
              codes.size(-1) == 128 && kscale.scalar_type() == at::kFloat,
          "dsa_key_write shapes");
    c10::cuda::CUDAGuard g(k.device());
    check_rc(xt_dsa_key_write(k.data_ptr(), ptr<const int64_t>(slot), codes.data_ptr(), ptr<float>(kscale),
                              int(k.size(0)), stream()),
             "dsa_key_write");
}

void dsa_index_decode(const Tensor &q, const Tensor &w, const Tensor &codes, const Tensor &kscale, const Tensor &base,
                      const Tensor &len, const Tensor &scores) {
    cuda_contig(q, "q");
    check(q.size(1) == 64 && q.size(2) == 128 && w.size(1) == 64 && base.scalar_type() == at::kLong &&
              len.scalar_type() == at::kInt && scores.scalar_type() == at::kFloat,
          "dsa_index_decode shapes");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_dsa_index_decode(q.data_ptr(), ptr<const float>(w), codes.data_ptr(), ptr<const float>(kscale),
                                 ptr<const int64_t>(base), ptr<const int32_t>(len), ptr<float>(scores),
                                 int(q.size(0)), int(scores.size(1)), stream()),
             "dsa_index_decode");
}

void dsa_index_tc(const Tensor &q8, const Tensor &w, const Tensor &codes, const Tensor &kscale, const Tensor &base,
                  const Tensor &len, const Tensor &scores, int64_t nq, const Tensor &err) {
    cuda_contig(q8, "q8");
    check(q8.scalar_type() == at::kByte && q8.size(1) == 64 && q8.size(2) == 128 && codes.size(-1) == 128 &&
              w.scalar_type() == at::kFloat && scores.scalar_type() == at::kFloat,
          "dsa_index_tc shapes");
    c10::cuda::CUDAGuard g(q8.device());
    check_rc(xt_dsa_index_tc(q8.data_ptr(), ptr<const float>(w), codes.data_ptr(), codes.size(0),
                             ptr<const float>(kscale), ptr<const int64_t>(base), ptr<const int32_t>(len),
                             ptr<float>(scores), int(q8.size(0)), int(scores.size(1)), int(nq), ptr<int>(err),
                             stream()),
             "dsa_index_tc");
}

void moe_grouped(const Tensor &x, const Tensor &codes, const Tensor &scales, const Tensor &gscale,
                 const Tensor &tiles, bool gate_up, int64_t I, int64_t fmt, const std::optional<Tensor> &route_w,
                 const Tensor &out, const Tensor &err, const std::optional<Tensor> &dst_rows) {
    cuda_contig(x, "x");
    cuda_contig(codes, "codes");
    cuda_contig(scales, "scales");
    cuda_contig(tiles, "tiles");
    check(x.scalar_type() == at::kBFloat16 && tiles.scalar_type() == at::kInt && tiles.size(1) == 4,
          "moe_grouped: bf16 x, int32 tiles [T, 4]");
    const int64_t R = x.size(0), K = x.size(1), slots = codes.size(0), N_rows = codes.size(1);
    check(codes.size(2) * 2 == K, "moe_grouped: codes [slots, N_rows, K/2]");
    if (gate_up)
        check(out.scalar_type() == at::kBFloat16 && out.size(0) == R && out.size(1) == I && N_rows == 2 * I,
              "moe_grouped gate_up: mid [R, I] bf16");
    else
        check(out.scalar_type() == at::kFloat && (dst_rows.has_value() || out.size(0) == R) &&
                  out.size(1) == N_rows && route_w.has_value(),
              "moe_grouped down: y [R, H] f32 (any row count with dst_rows) and route weights");
    if (dst_rows.has_value())
        check(!gate_up && dst_rows->scalar_type() == at::kInt && dst_rows->is_contiguous() && dst_rows->numel() == R,
              "moe_grouped: dst_rows int32 [R] (down only)");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_moe_grouped(x.data_ptr(), int(R), codes.data_ptr(), int(slots), ptr<const int32_t>(tiles),
                            int(tiles.size(0)), gate_up ? 1 : 0, int(K), int(N_rows), int(I), int(fmt),
                            scales.data_ptr(), ptr<const float>(gscale), optr<const float>(route_w),
                            optr<const int32_t>(dst_rows), gate_up ? out.data_ptr() : nullptr,
                            gate_up ? nullptr : ptr<float>(out),
                            int(out.size(1)), ptr<int>(err), stream()),
             "moe_grouped");
}

void topk_rows(const Tensor &scores, int64_t K, const Tensor &out, const std::optional<Tensor> &len) {
    cuda_contig(scores, "scores");
    check(scores.scalar_type() == at::kFloat && out.scalar_type() == at::kInt && out.size(0) == scores.size(0) &&
              out.size(1) == K,
          "topk_rows shapes");
    if (len.has_value())
        check(len->scalar_type() == at::kInt && len->is_contiguous() && len->numel() == scores.size(0),
              "topk_rows: len int32 [rows]");
    c10::cuda::CUDAGuard g(scores.device());
    check_rc(xt_topk_rows(ptr<const float>(scores), int(scores.size(0)), int(scores.size(1)), int(K),
                          optr<const int32_t>(len), ptr<int32_t>(out), stream()),
             "topk_rows");
}

void dsa_index_pf(const Tensor &q8, const Tensor &w, const Tensor &codes, const Tensor &kscale, int64_t row_base,
                  const Tensor &len, const Tensor &scores, int64_t splits, const Tensor &err) {
    cuda_contig(q8, "q8");
    cuda_contig(w, "w");
    cuda_contig(len, "len");
    cuda_contig(scores, "scores");
    check(q8.scalar_type() == at::kByte && q8.size(1) == 64 && q8.size(2) == 128 && codes.size(-1) == 128 &&
              w.scalar_type() == at::kFloat && scores.scalar_type() == at::kFloat && len.scalar_type() == at::kInt &&
              len.numel() == q8.size(0) && scores.size(0) >= q8.size(0),
          "dsa_index_pf shapes");
    check(row_base >= 0 && row_base + scores.size(1) <= codes.size(0), "dsa_index_pf: row outside the cache");
    c10::cuda::CUDAGuard g(q8.device());
    check_rc(xt_dsa_index_pf(q8.data_ptr(), ptr<const float>(w), codes.data_ptr(), codes.size(0),
                             ptr<const float>(kscale), row_base, ptr<const int32_t>(len), ptr<float>(scores),
                             int(q8.size(0)), int(scores.size(1)), int(splits), ptr<int>(err), stream()),
             "dsa_index_pf");
}

}  // namespace

// cudaLaunchHostFunc on a raw stream handle (graph capture records a host node); used by the row tables' lookup
extern "C" int xt_launch_host_fn(void *stream, void (*fn)(void *), void *arg) {
    return cudaLaunchHostFunc(static_cast<cudaStream_t>(stream), fn, arg) == cudaSuccess ? 0 : -1;
}

void mla_prep(const Tensor &in, int64_t q_lora, const Tensor &q_norm, const Tensor &kv_norm, const Tensor &pos,
              const Tensor &slot, double eps, double theta, const Tensor &q_out, const Tensor &codes,
              const Tensor &scales, const Tensor &rope, const std::optional<Tensor> &lat_out) {
    check(in.is_cuda() && in.dim() == 2 && in.stride(1) == 1 && in.scalar_type() == at::kBFloat16, "mla_prep input");
    check(pos.scalar_type() == at::kInt && slot.scalar_type() == at::kLong, "mla_prep: pos int32, slot int64");
    cuda_contig(q_out, "q_out");
    cuda_contig(codes, "codes");
    cuda_contig(scales, "scales");
    cuda_contig(rope, "rope");
    const int T = int(in.size(0));
    check(pos.numel() >= T && slot.numel() >= T && q_out.numel() >= int64_t(T) * q_lora, "mla_prep sizes");
    c10::cuda::CUDAGuard g(in.device());
    check_rc(xt_mla_prep(in.data_ptr(), int(in.stride(0)), int(q_lora), q_norm.data_ptr(), kv_norm.data_ptr(),
                         ptr<const int32_t>(pos), ptr<const int64_t>(slot), float(eps), float(theta), q_out.data_ptr(),
                         codes.data_ptr(), scales.data_ptr(), rope.data_ptr(), optr<void>(lat_out), T, stream()),
             "mla_prep");
}

void head_gemm(const Tensor &x, const Tensor &w, const Tensor &y, const std::optional<Tensor> &pos, int64_t rope_x,
               int64_t rope_y, int64_t rope_dims, double theta) {
    // x [T, heads, >= K] (last stride 1), w [heads, K, N], y [T, heads, >= N]
    check(x.is_cuda() && x.dim() == 3 && x.stride(2) == 1 && y.dim() == 3 && y.stride(2) == 1, "head_gemm layouts");
    cuda_contig(w, "w");
    check(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
          "head_gemm wants bf16");
    xt::HeadGemmParams p{};
    p.x = ptr<const __nv_bfloat16>(x);
    p.w = ptr<const __nv_bfloat16>(w);
    p.y = ptr<__nv_bfloat16>(y);
    p.xs_t = x.stride(0);
    p.xs_h = x.stride(1);
    p.ys_t = y.stride(0);
    p.ys_h = y.stride(1);
    p.T = int(x.size(0));
    p.K = int(w.size(1));
    p.N = int(w.size(2));
    check(x.size(1) == w.size(0) && y.size(1) == w.size(0), "head_gemm heads");
    p.pos = optr<const int32_t>(pos);
    p.rope_x = int(rope_x);
    p.rope_y = int(rope_y);
    p.rope_dims = int(rope_dims);
    p.theta = float(theta);
    if (p.rope_dims) check(p.pos && pos->scalar_type() == at::kInt, "head_gemm: int32 positions for the rotary part");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_head_gemm(&p, int(w.size(0)), stream()), "head_gemm");
}

void mx_quant_rows(const Tensor &x, const std::optional<Tensor> &src, const Tensor &x8, const Tensor &sfx) {
    cuda_contig(x, "x");
    cuda_contig(x8, "x8");
    cuda_contig(sfx, "sfx");
    const int64_t K = x8.size(-1), R = x8.numel() / K;
    check(x.scalar_type() == at::kBFloat16 && x.size(-1) == K && x8.scalar_type() == at::kByte &&
              sfx.scalar_type() == at::kByte && K % 128 == 0 && R % 128 == 0 && sfx.numel() >= R * (K / 32),
          "mx_quant_rows: x [*, K] bf16, x8 [R, K] u8 (R, K multiples of 128), sfx >= R * K / 32 bytes");
    if (src) check(src->is_contiguous() && src->scalar_type() == at::kInt && src->numel() == R, "mx_quant_rows src");
    else check(x.numel() == R * K, "mx_quant_rows: x [R, K] without src");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_mx_quant_rows(x.data_ptr(), optr<const int32_t>(src), int(R), int(K), x8.data_ptr(), sfx.data_ptr(),
                              stream()),
             "mx_quant_rows");
}

// y [M, N] BF16 (+ residual) = MXFP8 x8 [Mp, K] (rows past M dropped) . MXFP8 w8 [N, K]^T, both quantized by
// mx_quant_rows (scale atoms sfx, sfw)
void gemm_mx8(const Tensor &x8, const Tensor &sfx, int64_t M, const Tensor &w8, const Tensor &sfw,
              const std::optional<Tensor> &residual, const Tensor &y, const Tensor &err) {
    for (const Tensor *t : {&x8, &sfx, &w8, &sfw, &y}) cuda_contig(*t, "gemm_mx8 operand");
    const int64_t K = x8.size(-1), Mp = x8.numel() / K, N = w8.numel() / K;
    check(x8.scalar_type() == at::kByte && w8.scalar_type() == at::kByte && w8.size(-1) == K && K % 128 == 0 &&
              N % 128 == 0 && Mp % 128 == 0 && M > 0 && M <= Mp && sfx.numel() >= Mp * K / 32 &&
              sfw.numel() >= N * K / 32,
          "gemm_mx8: x8 [Mp, K], w8 [N, K] u8 (multiples of 128), scale atoms of both");
    check(y.scalar_type() == at::kBFloat16 && y.numel() == M * N, "gemm_mx8: y [M, N] bf16");
    if (residual)
        check(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16 && residual->numel() == M * N,
              "gemm_mx8: residual [M, N] bf16");
    check(err.is_cuda() && err.scalar_type() == at::kInt, "gemm_mx8 err int32");
    c10::cuda::CUDAGuard g(x8.device());
    check_rc(xt_gemm_mx8(x8.data_ptr(), sfx.data_ptr(), int(M), w8.data_ptr(), sfw.data_ptr(), int(N), int(K),
                         residual ? residual->data_ptr() : nullptr, y.data_ptr(), ptr<int>(err), stream()),
             "gemm_mx8");
}

// DeepSeek V4 mHC post-mix: x [M, H], res [M, 4, H] BF16, post [M, 4], comb [M, 4, 4] FP32 -> out [M, 4, H] BF16
void mhc_post(const Tensor &x, const Tensor &res, const Tensor &post, const Tensor &comb, const Tensor &out) {
    for (const Tensor *t : {&x, &res, &post, &comb, &out}) cuda_contig(*t, "mhc_post operand");
    const int64_t M = x.size(0), H = x.size(1);
    check(x.dim() == 2 && x.scalar_type() == at::kBFloat16 && res.scalar_type() == at::kBFloat16 &&
              res.numel() == M * 4 * H && out.scalar_type() == at::kBFloat16 && out.numel() == M * 4 * H &&
              post.scalar_type() == at::kFloat && post.numel() == M * 4 && comb.scalar_type() == at::kFloat &&
              comb.numel() == M * 16 && H % 8 == 0,
          "mhc_post: x [M, H], res / out [M, 4, H] bf16, post [M, 4], comb [M, 4, 4] f32, H % 8 == 0");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_mhc_post(x.data_ptr(), res.data_ptr(), ptr<float>(post), ptr<float>(comb), out.data_ptr(), int(M),
                         int(H), stream()),
             "mhc_post");
}

// DeepSeek V4 wo_a: o [T, G, D] BF16 view (unit stride along D) x W [G, R, D] (FP8 as uint8 with scale
// [G R / 32, D / 32] FP32, or BF16) -> out [T, G, R] BF16 view
void wo_a(const Tensor &o, const Tensor &w, const std::optional<Tensor> &scale, const Tensor &out) {
    check(o.is_cuda() && o.dim() == 3 && o.scalar_type() == at::kBFloat16 && o.stride(2) == 1,
          "wo_a: o [T, G, D] bf16 (unit stride along D)");
    cuda_contig(w, "w");
    const int64_t T = o.size(0), G = o.size(1), D = o.size(2);
    check(w.dim() == 3 && w.size(0) == G && w.size(2) == D, "wo_a: w [G, R, D]");
    const int64_t R = w.size(1);
    const bool fp8 = w.scalar_type() == at::kByte;
    check(fp8 || w.scalar_type() == at::kBFloat16, "wo_a: w uint8 (E4M3) or bf16");
    if (fp8) {
        check(scale && scale->is_cuda() && scale->scalar_type() == at::kFloat && scale->dim() == 2 &&
                  scale->size(0) == G * R / 32 && scale->size(1) == D / 32 && scale->stride(1) == 1,
              "wo_a: FP8 w needs scale [G R / 32, D / 32] f32");
    }
    check(out.is_cuda() && out.dim() == 3 && out.scalar_type() == at::kBFloat16 && out.size(0) == T &&
              out.size(1) == G && out.size(2) == R && out.stride(2) == 1,
          "wo_a: out [T, G, R] bf16 (unit stride along R)");
    c10::cuda::CUDAGuard g(o.device());
    check_rc(xt_wo_a(o.data_ptr(), o.stride(0), o.stride(1), fp8 ? w.data_ptr() : nullptr, fp8 ? nullptr : w.data_ptr(),
                     fp8 ? ptr<float>(*scale) : nullptr, fp8 ? int(scale->stride(0)) : 0, out.data_ptr(),
                     out.stride(0), out.stride(1), int(T), int(G), int(R), int(D), stream()),
             "wo_a");
}

// Qwen4-exp hyper-connection mix: x [rows, hc * hs], w_down [L, hc * hs], w_up [hc * hs, L] BF16 -> out [rows, hs];
// acc: FP32 workspace >= 16 * L
void hc_mix(const Tensor &x, const Tensor &wd, const Tensor &wu, const Tensor &acc, const Tensor &out, int64_t hc) {
    for (const Tensor *t : {&x, &wd, &wu, &acc, &out}) cuda_contig(*t, "hc_mix operand");
    const int64_t rows = x.size(0), K = x.size(1), L = wd.size(0);
    check(hc > 0 && K % hc == 0, "hc_mix: x [rows, hc * hs]");
    const int64_t hs = K / hc;
    check(x.scalar_type() == at::kBFloat16 && wd.scalar_type() == at::kBFloat16 && wu.scalar_type() == at::kBFloat16 &&
              wd.size(1) == K && wu.size(0) == K && wu.size(1) == L && acc.scalar_type() == at::kFloat &&
              acc.numel() >= 16 * L && out.scalar_type() == at::kBFloat16 && out.numel() == rows * hs,
          "hc_mix: shapes / dtypes");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_hc_mix(x.data_ptr(), wd.data_ptr(), wu.data_ptr(), ptr<float>(acc), out.data_ptr(), int(rows), int(hc),
                       int(hs), int(L), stream()),
             "hc_mix");
}

void moe_grouped_mx(const Tensor &x8, const Tensor &sfx, const Tensor &codes, const Tensor &scales,
                    const Tensor &gscale, const Tensor &tiles, bool gate_up, int64_t I,
                    const std::optional<Tensor> &route_w, const Tensor &out, const Tensor &err,
                    const std::optional<Tensor> &dst_rows) {
    cuda_contig(x8, "x8");
    cuda_contig(sfx, "sfx");
    cuda_contig(codes, "codes");
    cuda_contig(scales, "scales");
    cuda_contig(tiles, "tiles");
    check(x8.scalar_type() == at::kByte && tiles.scalar_type() == at::kInt && tiles.size(1) == 4,
          "moe_grouped_mx: u8 x8, int32 tiles [T, 4]");
    const int64_t R = x8.size(0), K = x8.size(1), slots = codes.size(0), N_rows = codes.size(1);
    check(codes.size(2) * 2 == K && scales.size(0) == slots && scales.size(1) == N_rows && scales.size(2) * 32 == K,
          "moe_grouped_mx: MXFP4 codes [slots, N_rows, K/2] and UE8M0 scales [slots, N_rows, K/32]");
    if (gate_up)
        check(out.scalar_type() == at::kBFloat16 && out.size(0) == R && out.size(1) == I && N_rows == 2 * I,
              "moe_grouped_mx gate_up: mid [R, I] bf16");
    else
        check(out.scalar_type() == at::kFloat && (dst_rows.has_value() || out.size(0) == R) &&
                  out.size(1) == N_rows && route_w.has_value(),
              "moe_grouped_mx down: y f32 and route weights");
    if (dst_rows.has_value())
        check(!gate_up && dst_rows->scalar_type() == at::kInt && dst_rows->numel() == R, "moe_grouped_mx dst_rows");
    c10::cuda::CUDAGuard g(x8.device());
    check_rc(xt_moe_grouped_mx(x8.data_ptr(), sfx.data_ptr(), int(R), codes.data_ptr(), scales.data_ptr(), int(slots),
                               ptr<const int32_t>(tiles), int(tiles.size(0)), gate_up ? 1 : 0, int(K), int(N_rows),
                               int(I), ptr<const float>(gscale), optr<const float>(route_w),
                               optr<const int32_t>(dst_rows), gate_up ? out.data_ptr() : nullptr,
                               gate_up ? nullptr : ptr<float>(out), int(out.size(1)), ptr<int>(err), stream()),
             "moe_grouped_mx");
}

int64_t pool_ring_create(int64_t capacity) {
    void *h = xt_pool_ring_create(int(capacity));
    check(h != nullptr, "pool_ring_create: mapped host or device allocation failed");
    return reinterpret_cast<int64_t>(h);
}

void pool_ring_destroy(int64_t h) { xt_pool_ring_destroy(reinterpret_cast<void *>(h)); }

int64_t pool_ring_post(int64_t h, int64_t seq, int64_t layer, int64_t expert, int64_t slot) {
    return xt_pool_ring_post(reinterpret_cast<void *>(h), seq, int(layer), int(expert), int(slot));
}

int64_t pool_ring_applied(int64_t h) { return xt_pool_ring_applied(reinterpret_cast<void *>(h)); }

void pool_ring_commit(int64_t h, const Tensor &tables, const Tensor &err) {
    cuda_contig(tables, "tables");
    check(tables.scalar_type() == at::kLong, "pool_ring_commit: tables int64 [layers] (device pointers)");
    c10::cuda::CUDAGuard g(tables.device());
    check_rc(xt_pool_ring_commit(reinterpret_cast<void *>(h), reinterpret_cast<int32_t *const *>(tables.data_ptr()),
                                 int(tables.numel()), ptr<int>(err), stream()),
             "pool_ring_commit");
}

void pool_ring_landed(int64_t h, int64_t seq, const Tensor &like) {
    c10::cuda::CUDAGuard g(like.device());
    check_rc(xt_pool_ring_landed(reinterpret_cast<void *>(h), seq, stream()), "pool_ring_landed");
}

void skinny_gemm(const Tensor &x, const Tensor &w, const std::optional<Tensor> &add, const Tensor &y,
                 const std::optional<Tensor> &part, int64_t splits, const Tensor &err) {
    cuda_contig(x, "x");
    cuda_contig(w, "w");
    cuda_contig(y, "y");
    const int64_t K = x.size(-1), M = x.numel() / K, N = w.size(0);
    check(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 &&
              w.size(1) == K && y.numel() == M * N && M >= 1 && M <= 32 && K % 64 == 0,
          "skinny_gemm: bf16 x [M <= 32, K % 64 == 0], w [N, K], y [M, N]");
    if (add) check(add->is_contiguous() && add->scalar_type() == at::kBFloat16 && add->numel() == M * N, "skinny add");
    if (splits > 1)
        check(part && part->is_contiguous() && part->scalar_type() == at::kFloat && part->numel() >= splits * M * N,
              "skinny_gemm: part [splits, M, N] f32");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_skinny_gemm(x.data_ptr(), w.data_ptr(), add ? add->data_ptr() : nullptr, y.data_ptr(),
                            optr<float>(part), int(M), int(N), int(K), int(splits), ptr<int>(err), stream()),
             "skinny_gemm");
}

void rope_heads(const Tensor &x, const Tensor &pos, double theta, const Tensor &out) {
    // x [T, H, d] and out [T, H, d] bf16 views with unit stride along d; pos int32 [T]
    check(x.is_cuda() && x.dim() == 3 && x.stride(2) == 1 && out.dim() == 3 && out.stride(2) == 1 &&
              x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
              x.sizes() == out.sizes() && pos.scalar_type() == at::kInt && pos.is_contiguous() &&
              pos.numel() == x.size(0),
          "rope_heads: x, out [T, H, d] bf16 (unit stride along d), pos int32 [T]");
    c10::cuda::CUDAGuard g(x.device());
    check_rc(xt_rope_heads(x.data_ptr(), x.stride(0), x.stride(1), ptr<const int32_t>(pos), float(theta),
                           out.data_ptr(), out.stride(0), out.stride(1), int(x.size(0)), int(x.size(1)),
                           int(x.size(2)), stream()),
             "rope_heads");
}

void dsa_quant_q(const Tensor &q, const Tensor &w, double w_scale, const Tensor &q8, const Tensor &w8) {
    cuda_contig(q, "q");
    cuda_contig(w, "w");
    cuda_contig(q8, "q8");
    cuda_contig(w8, "w8");
    check(q.scalar_type() == at::kBFloat16 && q.size(-1) == 128 && w.scalar_type() == at::kBFloat16 &&
              w.numel() * 128 == q.numel() && q8.scalar_type() == at::kByte && q8.numel() == q.numel() &&
              w8.scalar_type() == at::kFloat && w8.numel() == w.numel(),
          "dsa_quant_q: q [..., 128] bf16, w bf16 (one per row), q8 u8, w8 f32");
    c10::cuda::CUDAGuard g(q.device());
    check_rc(xt_dsa_quant_q(q.data_ptr(), w.data_ptr(), float(w_scale), q8.data_ptr(), ptr<float>(w8),
                            int(w.numel()), stream()),
             "dsa_quant_q");
}

void silu_mul(const Tensor &in, const Tensor &out) {
    cuda_contig(in, "in");
    cuda_contig(out, "out");
    check(in.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "silu_mul wants bf16");
    const int I = int(out.size(-1));
    const int T = int(out.numel() / I);
    check(in.numel() == int64_t(T) * 2 * I, "silu_mul shapes");
    c10::cuda::CUDAGuard g(in.device());
    check_rc(xt_silu_mul(in.data_ptr(), out.data_ptr(), T, I, stream()), "silu_mul");
}

TORCH_LIBRARY(xtier, m) {
    m.def("add_rmsnorm(Tensor x, Tensor(a!)? residual, Tensor w, Tensor(b!) out, float eps) -> ()");
    m.def("mla_prep(Tensor inp, int q_lora, Tensor q_norm, Tensor kv_norm, Tensor pos, Tensor slot, float eps, "
          "float theta, Tensor(a!) q_out, Tensor(b!) codes, Tensor(c!) scales, Tensor(d!) rope, Tensor(e!)? lat_out) "
          "-> ()");
    m.def("rope_heads(Tensor x, Tensor pos, float theta, Tensor(a!) out) -> ()");
    m.def("skinny_gemm(Tensor x, Tensor w, Tensor? add, Tensor(a!) y, Tensor(b!)? part, int splits, Tensor(c!) err) "
          "-> ()");
    m.def("mx_quant_rows(Tensor x, Tensor? src, Tensor(a!) x8, Tensor(b!) sfx) -> ()");
    m.def("mhc_post(Tensor x, Tensor res, Tensor post, Tensor comb, Tensor(a!) out) -> ()");
    m.def("wo_a(Tensor o, Tensor w, Tensor? scale, Tensor(a!) out) -> ()");
    m.def("hc_mix(Tensor x, Tensor wd, Tensor wu, Tensor(a!) acc, Tensor(b!) out, int hc) -> ()");
    m.def("gemm_mx8(Tensor x8, Tensor sfx, int M, Tensor w8, Tensor sfw, Tensor? residual, Tensor(a!) y, "
          "Tensor(b!) err) -> ()");
    m.def("pool_ring_create(int capacity) -> int", &pool_ring_create);
    m.def("pool_ring_destroy(int h) -> ()", &pool_ring_destroy);
    m.def("pool_ring_post(int h, int seq, int layer, int expert, int slot) -> int", &pool_ring_post);
    m.def("pool_ring_applied(int h) -> int", &pool_ring_applied);
    m.def("pool_ring_commit(int h, Tensor tables, Tensor(a!) err) -> ()");
    m.def("pool_ring_landed(int h, int seq, Tensor like) -> ()");
    m.def("moe_grouped_mx(Tensor x8, Tensor sfx, Tensor codes, Tensor scales, Tensor gscale, Tensor tiles, "
          "bool gate_up, int I, Tensor? route_w, Tensor(a!) out, Tensor(b!) err, Tensor? dst_rows=None) -> ()");
    m.def("dsa_quant_q(Tensor q, Tensor w, float w_scale, Tensor(a!) q8, Tensor(b!) w8) -> ()");
    m.def("head_gemm(Tensor x, Tensor w, Tensor(a!) y, Tensor? pos, int rope_x, int rope_y, int rope_dims, "
          "float theta) -> ()");
    m.def("silu_mul(Tensor inp, Tensor(a!) out) -> ()");
    m.def("qk_norm_rope_kv(Tensor qkv, Tensor? q_norm, Tensor? k_norm, Tensor pos, Tensor batch, Tensor(a!) q, "
          "Tensor(b!) k_cache, Tensor(c!) v_cache, int hq, int hkv, float theta, float eps, Tensor? slots=None) -> ()");
    m.def("attn_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seqlens, Tensor(a!) out, Tensor(b!) ws_o, "
          "Tensor(c!) ws_ml, Tensor(d!) counters, int splits, float scale) -> ()");
    m.def("moe_route(Tensor x, Tensor wr, Tensor? bias, Tensor? corr, Tensor? table, Tensor? shared_slots, "
          "Tensor(a!) ids, Tensor(b!) w, Tensor(c!) slots, Tensor(d!) ws_logits, Tensor(e!) ws_count, int k, int mode, "
          "int n_group, int topk_group, bool renorm, float scale, int layer, int mailbox, Tensor? active=None, "
          "Tensor? logits_in=None, Tensor? cold_index=None, int share_min=0, int host_base=0, Tensor(f!)? claim=None, "
          "Tensor(g!)? claim_list=None, Tensor(h!)? claim_count=None, int stage_max=0, int stage_slot0=0) -> ()");
    m.def("gemv(Tensor x, Tensor w, Tensor? add, Tensor(a!) out) -> ()");
    m.def("fp8_rows(Tensor tab, Tensor scales, Tensor? ids, int lo, int hi, int blk, Tensor(a!) out) -> ()");
    m.def("gemv_fp8(Tensor x, Tensor w, Tensor s, Tensor? add, Tensor(a!) out) -> ()");
    m.def("fp8_dequant(Tensor w, Tensor s, Tensor(a!) out) -> ()");
    m.def("gemm_tc_f32(Tensor a, Tensor b, Tensor(a!) out, Tensor(b!) err) -> ()");
    m.def("gather_rows(Tensor x, Tensor src, Tensor(a!) X) -> ()");
    m.def("route_combine(Tensor Ya, Tensor da, Tensor? Yb, Tensor? db, Tensor? add, Tensor(a!) out) -> ()");
    m.def("spec_truncate(Tensor(a!) q, Tensor tokens, Tensor? topk, Tensor(b!) flags, float threshold) -> ()");
    m.def("gemm_tc(Tensor a, Tensor b, Tensor? residual, Tensor(a!) out, Tensor(b!) err) -> ()");
    m.def("ep_moe(Tensor x, Tensor ids, Tensor w, Tensor peer, Tensor(a!) state, Tensor(b!) mid, Tensor w13, "
          "Tensor s13, Tensor g13, Tensor w2, Tensor s2, Tensor g2, Tensor? add, Tensor(c!) out, Tensor(d!) err, "
          "int W, int rank, int E, int fmt, int R, int[] offsets, float timeout_s, int phases, Tensor? slots=None, "
          "int spr=0, int mailbox=0, Tensor? st_w13=None, Tensor? st_s13=None, Tensor? st_w2=None, "
          "Tensor? st_s2=None, Tensor? st_g13=None, Tensor? st_g2=None, int stage_base=0) -> ()");
    m.def("qsa_kv_write(Tensor x, Tensor slots, Tensor(a!) codes, Tensor(b!) scales) -> ()");
    m.def("qsa_decode(Tensor q, Tensor idx, Tensor kc, Tensor ks, Tensor vc, Tensor vs, Tensor(a!) part_o, "
          "Tensor(b!) part_ml, Tensor(c!) out, float scale) -> ()");
    m.def("ep_stage(Tensor claim_list, Tensor(a!) claim, Tensor(b!) claim_count, Tensor(c!) done, Tensor cold_index, "
          "int[] bases, int stride, int[] piece_off, int[] piece_bytes, Tensor(d!) w13, Tensor(e!) s13, "
          "Tensor(f!) w2, Tensor(g!) s2, Tensor(h!) g13, Tensor(i!) g2, Tensor src_g13, Tensor src_g2, int I, int H, "
          "int fmt, int chunks) -> ()");
    m.def("l2_prefetch(Tensor ptrs, Tensor bytes, int ctas) -> ()");
    m.def("dsa_key_write(Tensor k, Tensor slot, Tensor(a!) codes, Tensor(b!) kscale) -> ()");
    m.def("dsa_index_decode(Tensor q, Tensor w, Tensor codes, Tensor kscale, Tensor base, Tensor len, "
          "Tensor(a!) scores) -> ()");
    m.def("topk_rows(Tensor scores, int K, Tensor(a!) out, Tensor? len=None) -> ()");
    m.def("dsa_index_pf(Tensor q8, Tensor w, Tensor codes, Tensor kscale, int row_base, Tensor len, "
          "Tensor(a!) scores, int splits, Tensor(b!) err) -> ()");
    m.def("moe_grouped(Tensor x, Tensor codes, Tensor scales, Tensor gscale, Tensor tiles, bool gate_up, int I, "
          "int fmt, Tensor? route_w, Tensor(a!) out, Tensor(b!) err, Tensor? dst_rows=None) -> ()");
    m.def("dsa_index_tc(Tensor q8, Tensor w, Tensor codes, Tensor kscale, Tensor base, Tensor len, Tensor(a!) scores, "
          "int nq, Tensor(b!) err) -> ()");
    m.def("mla_kv_write(Tensor lat, Tensor slot, Tensor(a!) codes, Tensor(b!) scales, Tensor(c!) rope) -> ()");
    m.def("attn_prefill(Tensor q, Tensor k, Tensor v, Tensor(a!) out, int row, int start, float scale, "
          "Tensor(b!) err, Tensor? tree_mask=None) -> ()");
    m.def("mla_flash(Tensor q, Tensor idx, Tensor codes, Tensor scales, Tensor rope, Tensor(a!)? part_o, "
          "Tensor(b!)? part_ml, Tensor(c!) out, float scale, int splits, Tensor(d!) err, Tensor? q_rope=None) -> ()");
    m.def("mla_decode(Tensor q, Tensor idx, Tensor codes, Tensor scales, Tensor rope, Tensor(a!) kg, Tensor(b!) vt, "
          "Tensor(c!) part_o, Tensor(d!) part_ml, Tensor(e!) out, float scale, Tensor(f!) err) -> ()");
    m.def("gemm_rs(Tensor a, Tensor b, Tensor peer, Tensor(a!) state, Tensor? residual, Tensor(b!) out, "
          "Tensor(c!) err, int W, int rank, int[] offsets, float timeout_s) -> ()");
    m.def("ag_gemm(Tensor a_shard, Tensor b, Tensor peer, int local_base, Tensor(a!) state, Tensor(b!) out, "
          "Tensor(c!) err, int W, int rank, int[] offsets, float timeout_s) -> ()");
    m.def("moe_gate_up(Tensor x, Tensor slots, Tensor w13, Tensor s13, Tensor g13, Tensor(a!) mid, int fmt, "
          "float limit, float alpha, float beta, Tensor? peer=None, int spr=0, Tensor? host=None, "
          "int host_base=0) -> ()");
    m.def("moe_down(Tensor mid, Tensor slots, Tensor w, Tensor w2, Tensor s2, Tensor g2, Tensor? add, Tensor(a!) out, "
          "Tensor(b!)? out_f32, Tensor(c!)? gpu_part, int fmt, int mailbox, Tensor? peer=None, int spr=0, "
          "Tensor? host=None, int host_base=0) -> ()");
}

TORCH_LIBRARY_IMPL(xtier, CUDA, m) {
    m.impl("add_rmsnorm", &add_rmsnorm);
    m.impl("mla_prep", &mla_prep);
    m.impl("head_gemm", &head_gemm);
    m.impl("rope_heads", &rope_heads);
    m.impl("skinny_gemm", &skinny_gemm);
    m.impl("pool_ring_commit", &pool_ring_commit);
    m.impl("pool_ring_landed", &pool_ring_landed);
    m.impl("mx_quant_rows", &mx_quant_rows);
    m.impl("mhc_post", &mhc_post);
    m.impl("wo_a", &wo_a);
    m.impl("hc_mix", &hc_mix);
    m.impl("gemm_mx8", &gemm_mx8);
    m.impl("moe_grouped_mx", &moe_grouped_mx);
    m.impl("dsa_quant_q", &dsa_quant_q);
    m.impl("silu_mul", &silu_mul);
    m.impl("qk_norm_rope_kv", &qk_norm_rope_kv);
    m.impl("attn_decode", &attn_decode);
    m.impl("moe_route", &moe_route);
    m.impl("ep_stage", &ep_stage);
    m.impl("qsa_kv_write", &qsa_kv_write);
    m.impl("qsa_decode", &qsa_decode);
    m.impl("moe_gate_up", &moe_gate_up);
    m.impl("moe_down", &moe_down);
    m.impl("gemv", &gemv);
    m.impl("fp8_rows", &fp8_rows);
    m.impl("gemv_fp8", &gemv_fp8);
    m.impl("fp8_dequant", &fp8_dequant);
    m.impl("gemm_tc_f32", &gemm_tc_f32);
    m.impl("gather_rows", &gather_rows);
    m.impl("route_combine", &route_combine);
    m.impl("spec_truncate", &spec_truncate);
    m.impl("gemm_tc", &gemm_tc);
    m.impl("ep_moe", &ep_moe);
    m.impl("gemm_rs", &gemm_rs);
    m.impl("ag_gemm", &ag_gemm);
    m.impl("l2_prefetch", &l2_prefetch);
    m.impl("mla_kv_write", &mla_kv_write);
    m.impl("mla_decode", &mla_decode);
    m.impl("attn_prefill", &attn_prefill);
    m.impl("mla_flash", &mla_flash);
    m.impl("dsa_key_write", &dsa_key_write);
    m.impl("dsa_index_decode", &dsa_index_decode);
    m.impl("topk_rows", &topk_rows);
    m.impl("moe_grouped", &moe_grouped);
    m.impl("dsa_index_tc", &dsa_index_tc);
    m.impl("dsa_index_pf", &dsa_index_pf);
}
