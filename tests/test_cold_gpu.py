"""Cold experts in the model: XTIER_COLD with half of each layer's CPU-tier experts kept only in the drive store; the
CPU engine reads its misses from the store inside mailbox calls; logits match the fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_model_with_cold_store(cuda_ops, tmp_path, monkeypatch):
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    monkeypatch.setenv('XTIER_COLD', '1')
    monkeypatch.setenv('XTIER_COLD_DIR', f'{tmp_path / "d0"},{tmp_path / "d1"}')
    monkeypatch.setenv('XTIER_COLD_FRACTION', '0.5')
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128, experts=16, top_k=4)
    mb = Mailbox(cfg.hidden, timeout_s=20.0)
    model = Qwen3MoeModel(cfg, device='cuda', seed=6, hot_fraction=0.25, synthetic_experts=False,
                          engine_threads=2, mailbox=mb)
    assert model.cold is not None and model.engines and model.engines[0].shape()['slots'] == 8
    mb.start()
    try:
        prompt = torch.randint(0, cfg.vocab, (12,), generator=torch.Generator().manual_seed(7)).cuda()
        st = model.alloc_state(1, 32)
        _, lp = model.prefill(st, prompt, return_logits=True)   # 12 tokens: the decode path and the mailbox
        torch.cuda.synchronize()
        mb.check()
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
        assert sum(e.cold_stats()['reads'] for e in model.engines) > 0
        assert model.cold.stats()['bytes_read'] > 0
    finally:
        mb.stop()
        model.cold.close()


def test_cold_mode_grouped_prefill_without_host_copy(cuda_ops, tmp_path, monkeypatch):
    """Grouped GPU prefill of a cold-mode model: no host copy of any layer is kept; each layer's non-GPU experts are
    staged from the engine's RAM slots and the drives (the next layer read ahead while this one computes), also
    after GPU-slot swaps sourced from the same tier; logits match the fp32 reference rebuilt from the store."""
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    monkeypatch.setenv('XTIER_COLD', '1')
    monkeypatch.setenv('XTIER_COLD_DIR', f'{tmp_path / "d0"},{tmp_path / "d1"}')
    monkeypatch.setenv('XTIER_COLD_FRACTION', '0.5')
    monkeypatch.setenv('XTIER_COLD_UNITS', '3')
    monkeypatch.setenv('XTIER_GPU_PREFILL_MIN', '16')
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128, experts=16, top_k=4)
    model = Qwen3MoeModel(cfg, device='cuda', seed=9, hot_fraction=0.25, synthetic_experts=False, engine_threads=2)
    try:
        assert all(L['moe'].host is None and L['moe'].cold_prefill is not None for L in model.layers)
        prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(5)).cuda()
        st = model.alloc_state(1, 64)
        _, lp = model.prefill(st, prompt, return_logits=True)
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
        stats = [L['moe'].cold_prefill.stats for L in model.layers]
        assert all(s['fills'] == 1 for s in stats)
        assert sum(s['from_drive'] for s in stats) > 0 and sum(s['from_ram'] for s in stats) > 0
        for L in model.layers:            # swaps read the incoming expert from the engine or the drives
            moe = L['moe']
            hot = moe.resident()
            cold = [e for e in range(moe.E) if e not in hot]
            moe.swap(cold[-1], hot[0])
        torch.cuda.synchronize()
        st = model.alloc_state(1, 64)
        _, lp = model.prefill(st, prompt, return_logits=True)
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
    finally:
        model.cold.close()
