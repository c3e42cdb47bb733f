"""Process-group setup: RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* from the environment (torchrun), NCCL for the
device group (with a short timeout so ranks that wait for one another end with an error) and gloo for host-side
exchanges (handle bytes, shapes)."""
from __future__ import annotations

import dataclasses
import os
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclasses.dataclass
class DistEnv:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device | None = None
    cpu_group: object = None

    @property
    def enabled(self) -> bool:
        return self.world > 1


_env = DistEnv()


def init(backend: str | None = None, timeout_s: float = 300.0) -> DistEnv:
    """Initializes once; a single process (no WORLD_SIZE) gets world 1 and no process group."""
    global _env
    if _env.device is not None:
        return _env
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', str(rank)))
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    os.environ.setdefault('MASTER_PORT', '29531')
    cuda = torch.cuda.is_available()
    device = torch.device('cuda', local) if cuda else torch.device('cpu')
    if cuda:
        torch.cuda.set_device(device)
    cpu_group = None
    if world > 1 and not dist.is_initialized():
        be = backend or ('nccl' if cuda else 'gloo')
        kw = dict(backend=be, timeout=timedelta(seconds=timeout_s))
        if be == 'nccl':
            kw['device_id'] = device
        dist.init_process_group(**kw)
        cpu_group = dist.new_group(backend='gloo', timeout=timedelta(seconds=timeout_s)) if be == 'nccl' else \
            dist.group.WORLD
    elif world > 1:   # the caller made the process group: host exchanges still need a gloo group (collective call)
        cpu_group = dist.new_group(backend='gloo', timeout=timedelta(seconds=timeout_s)) \
            if dist.get_backend() == 'nccl' else dist.group.WORLD
    _env = DistEnv(rank, world, local, device, cpu_group)
    return _env


def get() -> DistEnv:
    return _env


def all_gather_bytes(data: bytes, group=None) -> list[bytes]:
    """Every rank's bytes (equal lengths), through the host group."""
    env = get()
    if env.world == 1:
        return [data]
    t = torch.frombuffer(bytearray(data), dtype=torch.uint8)
    out = [torch.empty_like(t) for _ in range(env.world)]
    dist.all_gather(out, t, group=group or env.cpu_group)
    return [bytes(o.numpy()) for o in out]


def barrier():
    if get().world > 1:
        dist.barrier(group=get().cpu_group)
