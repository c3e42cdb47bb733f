"""Serving metrics snapshot and its Prometheus text form (fake mailbox and model)."""
import numpy as np

from xtier_b200.utils.metrics import prometheus_text, snapshot


class _MB:
    def stats(self):
        return dict(calls=10.0, mean_us=55.5, cpu_error=0.0, gpu_error=0.0, wall_us=1.0, seq=10.0)

    def layer_stats(self, layer, E):
        return np.zeros(E, np.float32), dict(calls=4.0, cpu_us=200.0, cpu_routes=6.0, gpu_routes=18.0)


class _Moe:
    def __init__(self, i):
        self.layer, self.E, self.mailbox = i, 8, object()


class _Pol:
    total_swaps = 3


class _Model:
    layers = [{'moe': _Moe(0)}, {'moe': _Moe(1)}]
    policy = _Pol()


def test_snapshot_and_prometheus():
    snap = snapshot(_Model(), _MB(), {'requests': 2, 'tokens': 64})
    assert snap['requests_total'] == 2 and snap['mailbox_calls_total'] == 10.0 and snap['swaps_total'] == 3
    assert snap['layers'][1]['hit_rate'] == 0.75 and snap['layers'][0]['cpu_us_per_call'] == 50.0
    text = prometheus_text(snap)
    assert '# TYPE xtier_tokens_total counter' in text and 'xtier_tokens_total 64' in text
    assert 'xtier_layer_hit_rate{layer="1"} 0.75' in text
    assert 'xtier_mailbox_cpu_us_mean 55.5' in text
