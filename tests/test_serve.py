

def test_deepseek_build_caps_hbm_slots(monkeypatch):
    """The DeepSeek server's HBM slots: the --hot share, capped by what fits beside the dense weights (fakes for the
    model, mailbox and decode runtime; no GPU)."""
    import argparse

    import torch

    from xtier_b200 import serve
    from xtier_b200.engine import mailbox as mbmod
    from xtier_b200.models import deepseek_v3 as dsm
    from xtier_b200.runtime import decode as dec
    seen = {}

    class FakeModel:
        def __init__(self, cfg, **kw):
            seen.update(kw)
            self.cfg = cfg

    class FakeGen:
        def __init__(self, model, batch, max_len):
            self.max_len, self.sampling = max_len, False

    class FakeBackend:
        def __init__(self, model, gen, tok, mailbox, prefix_cache=True):
            self.prefix_cache, self.mailbox = prefix_cache, mailbox

        def prefill(self, ids):
            return 0

    class FakeMailbox:
        def __init__(self, hidden):
            pass

        def start(self):
            pass

    monkeypatch.setattr(dsm, 'DeepSeekV3Model', FakeModel)
    monkeypatch.setattr(dec, 'Generator', FakeGen)
    monkeypatch.setattr(mbmod, 'Mailbox', FakeMailbox)
    monkeypatch.setattr(serve, 'GenBackend', FakeBackend)
    cfg = dsm.DeepSeekV3Config(layers=61, attn='mla')
    per = cfg.expert_bytes() * cfg.moe_layers()
    free = cfg.dense_bytes() + (6 << 30) + 112 * per + per // 2        # room for 112 experts per layer
    monkeypatch.setattr(torch.cuda, 'mem_get_info', lambda *a: (free, free))
    stages = serve.Stages(emit=lambda *a, **k: None)
    args = argparse.Namespace(checkpoint=None, sampling=False, batch=1, recall=None, layers=None, hot=0.56, seed=0,
                              max_len=1024)
    be = serve.build_deepseek(args, stages)
    assert seen['gpu_experts'] == 112 and be.mailbox is not None and not be.prefix_cache
    args.hot = 0.25
    serve.build_deepseek(args, stages)
    assert seen['gpu_experts'] == 64
