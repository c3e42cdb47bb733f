"""Draft trees on the GPU: the prefill attention kernel with a tree mask against an fp32 reference, and speculative
decoding over trees (draft chain plus Recall copies) producing exactly the target's greedy tokens."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tree_mask_attention_vs_fp32(cuda_ops):
    from xtier_b200 import ops
    from xtier_b200.runtime.tree import build_tree
    Hq, Hkv, start = 8, 2, 300
    tree = build_tree(5, [([1, 2, 3, 4], [1.0] * 4), ([1, 6, 7], [0.9] * 3), ([8, 9], [0.7] * 2)], budget=16)
    n = tree.n
    g = torch.Generator(device='cuda').manual_seed(3)
    k = torch.randn(1, Hkv, 512, 128, device='cuda', generator=g).bfloat16()
    v = torch.randn(1, Hkv, 512, 128, device='cuda', generator=g).bfloat16()
    q = torch.randn(n, Hq, 128, device='cuda', generator=g).bfloat16()
    words = torch.as_tensor(tree.ancestor_words()).cuda()
    out = ops.attn_prefill(q, k, v, 0, start, 1 / math.sqrt(128), tree_mask=words)
    torch.cuda.synchronize()
    vis = torch.zeros(n, start + n, dtype=torch.bool)
    vis[:, :start] = True
    for i in range(n):
        for j in tree.path(i):
            vis[i, start + j] = True
    kk = k[0, :, :start + n].float().repeat_interleave(Hq // Hkv, 0)
    vv = v[0, :, :start + n].float().repeat_interleave(Hq // Hkv, 0)
    s = torch.einsum('thd,hnd->htn', q.float(), kk) / math.sqrt(128)
    s = s.masked_fill(~vis.cuda()[None], float('-inf'))
    ref = torch.einsum('htn,hnd->thd', torch.softmax(s, -1), vv)
    assert float((out.float() - ref).norm() / ref.norm()) < 1e-2


def _tiny(seed, layers=2):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128)
    cfg.layers = layers
    return Qwen3MoeModel(cfg, device='cuda', seed=seed, hot_fraction=1.0, synthetic_experts=False)


def _greedy(model, prompt, n):
    st = model.alloc_state(1, 256)
    out, nxt, pos = [], model.prefill(st, prompt), prompt.shape[0]
    for _ in range(n):
        out.append(int(nxt))
        nxt = model.prefill(st, nxt.view(1), start=pos)
        pos += 1
    return out


def test_tree_speculation_equals_target_greedy(cuda_ops):
    from xtier_b200 import recall
    from xtier_b200.runtime.speculative import SpeculativeDecoder
    target = _tiny(31)
    draft = _tiny(31, layers=1)
    prompt = torch.randint(0, target.cfg.vocab, (20,), generator=torch.Generator().manual_seed(5)).cuda()
    want = _greedy(target, prompt, 40)
    # the record holds the prompt followed by the target's own continuation with a wrong stretch in the middle:
    # copies land, then miss, and the draft chain competes in the same trees
    bad = list(want)
    bad[18:22] = [(t + 1) % target.cfg.vocab for t in bad[18:22]]
    rec = recall.Record()
    rec.add(prompt.tolist() + bad)
    eng = recall.RecallEngine(rec, gamma=8, min_n=0.0)
    sd = SpeculativeDecoder(target, draft, steps=3, threshold=0.0, max_len=256, recall=eng, tree=True, tree_nodes=16)
    got = sd.generate(prompt, 40)
    assert got == want, (got, want)
    assert sd.stats['tree_rounds'] > 0 and sd.stats['forwards'] < 40
    assert sd.stats['tree_accepted'] > 0
