"""Hot slots spread over 2 GPUs (one process per GPU): routes to an expert that only the other GPU holds are computed
from its pool over NVLink, the rest go to the CPU tier; the model's logits match the fp32 reference on both ranks."""
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR='127.0.0.1',
                          MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        from xtier_b200 import ops
        from xtier_b200.engine.mailbox import Mailbox
        from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
        from xtier_b200.parallel import dist as xdist
        xdist.init(timeout_s=60)
        ops.load()
        cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128, experts=16, top_k=4)
        mb = Mailbox(cfg.hidden, timeout_s=20.0)
        model = Qwen3MoeModel(cfg, device='cuda', seed=3, hot_fraction=0.25, synthetic_experts=False,
                              engine_threads=2, mailbox=mb, peer=True)
        mb.start()
        prompt = torch.randint(0, cfg.vocab, (12,), generator=torch.Generator().manual_seed(10 + rank)).cuda()
        st = model.alloc_state(1, 32)
        _, lp = model.prefill(st, prompt, return_logits=True)   # 12 tokens: the decode-path MoE kernels
        torch.cuda.synchronize()
        mb.check()
        moe = model.layers[0]['moe']
        slots = moe.slots[:12, :cfg.top_k].cpu()
        remote = int(((slots >= 0) & (slots // moe.spr != rank)).sum())
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        xdist.barrier()
        mb.stop()
        q.put((rank, rel, remote, None))
        torch.distributed.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


def test_peer_slots_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, rel, remote, err in results:
        assert err is None, err
        assert rel < 3e-2, (rank, rel)
    assert sum(r[2] for r in results) > 0     # some routes were served from the other GPU's pool
