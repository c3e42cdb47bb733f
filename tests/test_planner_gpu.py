"""Planner probes on the GPU: graph-replayed decode MoE timings, the measured mailbox round trip (a layer without GPU
slots whose route goes to a tiny expert on the CPU engine, minus that expert's engine time), and the coefficients
the planner reads."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_probes_measure_gpu_and_mailbox(cuda_ops):
    from xtier_b200.planner import probe
    g = probe.probe_gpu(512, 256, reps=10)
    assert [k for k, _ in g] == [1, 2, 4, 8] and all(t > 0 for _, t in g)
    mb = probe.probe_mailbox(512, threads=2, reps=10)
    assert mb['call_us'] > mb['engine_us'] > 0
    out = probe.measure(512, 256, threads=2)
    co = out['coeffs']
    assert co['c0'] >= 1.0 and co['g0'] > 0 and 'mailbox' in out['samples']
    if torch.cuda.device_count() >= 2:
        assert co['p1'] > 0 and out['samples']['peer']['gbs'] > 0
    # PCIe staging: the ep_stage copy from registered engine memory (bytes checked inside the probe), 1-8 experts
    pc = out['samples']['pcie']
    assert [n for n, _ in pc] == [1, 2, 4, 8] and all(t > 0 for _, t in pc) and co['h1'] >= 0.1
