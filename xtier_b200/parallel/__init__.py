"""Multi-GPU: one process per GPU (torch.distributed, NCCL for the plumbing), symmetric peer memory, expert-parallel
MoE with in-kernel NVLink dispatch/combine (ep.py), and the NCCL all-to-all baseline."""
from .dist import DistEnv, init, get  # noqa: F401
