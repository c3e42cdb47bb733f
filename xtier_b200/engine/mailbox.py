"""CPU<->GPU mailbox (host side in csrc/mailbox/mailbox.cpp, device side in csrc/cuda/moe_decode.cu).

A `Mailbox` owns one mapped pinned slot, its device state and a dispatcher thread that runs the registered CPU engine
plans. The GPU MoE kernels receive `mailbox.handle` and talk to the dispatcher through the slot; nothing on this path
allocates or synchronizes, so a decode step with CPU experts can be captured in a CUDA graph. Each GPU-side wait has a
deadline (`timeout_s`); `check()` raises when a wait ran out or the CPU engine failed.

Reference parity: xtier/engine/__init__.py:328-370 (Mailbox), csrc/include/xtier_mailbox.h:11-79.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .. import config


class MailboxError(RuntimeError):
    pass


def _lib():
    from .. import ops
    L = ops.cdll()
    if not getattr(L, '_xt_mb_typed', False):
        L.xt_mailbox_create.restype = C.c_void_p
        L.xt_mailbox_create.argtypes = [C.c_int, C.c_double]
        L.xt_mailbox_register.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        L.xt_mailbox_start.argtypes = [C.c_void_p, C.c_int, C.c_float]
        L.xt_mailbox_stop.argtypes = [C.c_void_p]
        L.xt_mailbox_stats.argtypes = [C.c_void_p, C.c_void_p]
        L.xt_mailbox_layer_stats.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.xt_mailbox_clear_errors.argtypes = [C.c_void_p]
        L.xt_mailbox_host_ptrs.argtypes = [C.c_void_p, C.c_void_p]
        L.xt_mailbox_destroy.argtypes = [C.c_void_p]
        L.xt_mailbox_error.restype = C.c_char_p
        L._xt_mb_typed = True
    return L


def dispatcher_cpu() -> int:
    cpu = config.get('XTIER_DISPATCH_CPU')
    if cpu is not None and cpu >= 0:
        return cpu
    cpus = sorted(os.sched_getaffinity(0))
    return cpus[-1] if cpus else -1


class Mailbox:
    def __init__(self, hidden: int, timeout_s: float | None = None):
        L = _lib()
        self.hidden = hidden
        t = config.get('XTIER_CPU_TIMEOUT_S') if timeout_s is None else timeout_s
        self.handle = L.xt_mailbox_create(hidden, float(t))
        if not self.handle:
            raise MailboxError(L.xt_mailbox_error().decode())
        self._plans = {}
        self.started = False

    def register(self, layer: int, engine):
        """Routes of `layer` that miss the GPU run on `engine` (a CpuEngine)."""
        self._plans[layer] = engine
        _lib().xt_mailbox_register(self.handle, layer, engine.plan, engine.E)

    def start(self, cpu: int | None = None, decay: float = 0.999):
        if not self.started:
            _lib().xt_mailbox_start(self.handle, dispatcher_cpu() if cpu is None else cpu, decay)
            self.started = True

    def stop(self):
        if self.started:
            _lib().xt_mailbox_stop(self.handle)
            self.started = False

    def stats(self) -> dict:
        out = (C.c_double * 8)()
        _lib().xt_mailbox_stats(self.handle, out)
        return dict(calls=out[0], mean_us=out[1], cpu_error=out[2], gpu_error=out[3], wall_us=out[4], seq=out[5])

    def layer_stats(self, layer: int, experts: int):
        counts = np.zeros(experts, dtype=np.float32)
        st = (C.c_double * 4)()
        if _lib().xt_mailbox_layer_stats(self.handle, layer, counts.ctypes.data, st) < 0:
            raise KeyError(layer)
        return counts, dict(calls=st[0], cpu_us=st[1], cpu_routes=st[2], gpu_routes=st[3])

    def check(self):
        """Raises if a GPU wait timed out or a CPU engine call failed since the last check."""
        s = self.stats()
        if s['gpu_error'] or s['cpu_error']:
            _lib().xt_mailbox_clear_errors(self.handle)
            what = 'a GPU wait for the CPU timed out' if s['gpu_error'] else 'a CPU engine call failed'
            raise MailboxError(f'xtier_b200 mailbox: {what} (calls so far {int(s["calls"])})')

    def close(self):
        if getattr(self, 'handle', None):
            _lib().xt_mailbox_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
