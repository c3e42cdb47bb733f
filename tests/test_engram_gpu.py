"""Hashed bigram NVMe rows in the model: the prompt's rows in prefill and the decode token's rows looked up inside the
captured decode graph; logits match the fp32 reference forward of the whole sequence at every step."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bigram_rows_in_prefill_and_decode_graph(cuda_ops, tmp_path):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    from xtier_b200.tables import RowStore, write_table
    from xtier_b200.tables.engram import BigramTable
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128)
    model = Qwen3MoeModel(cfg, device='cuda', seed=4, hot_fraction=1.0, synthetic_experts=False)
    rows, dim = 5000, 128                                      # narrower than the hidden size: a projection
    data = torch.from_numpy((np.random.default_rng(2).standard_normal((rows, dim)) * 0.5).astype(np.float32))
    bf = data.bfloat16()
    segs = write_table(tmp_path / 'bigram', bf.view(torch.uint8).numpy().reshape(rows, dim * 2), None, segments=2)
    store = RowStore(segs, dim * 2, 0, io_threads=2, cache_rows=128)
    proj = (torch.randn(cfg.hidden, dim, generator=torch.Generator().manual_seed(3)) * 0.1).bfloat16()
    model.attach_bigram(BigramTable(store, rows, dim, cfg.hidden, batch=1, device='cuda', seed=9, proj=proj))
    prompt = torch.randint(0, cfg.vocab, (1, 10), generator=torch.Generator().manual_seed(5))
    gen = Generator(model, batch=1, max_len=64)
    gen.prefill(prompt)
    gen.capture()
    seq = prompt[0].tolist() + [int(gen.buf['tokens'][0])]
    for _ in range(3):
        gen.host_tokens.copy_(gen.buf['tokens'].cpu())
        nxt = int(gen.decode_one()[0])
        gen.check()
        ref = model.reference_logits(torch.tensor(seq).cuda())
        got = gen.buf['logits'][0].float()
        rel = float((got - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
        seq.append(nxt)
    gen.graph = None
    store.close()
