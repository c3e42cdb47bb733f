"""A smaller GPU on this one: holds all of the GPU's free memory except FREE_MIB (one allocation through torch) until
process WATCH_PID exits, so every allocator of a server started next to it (torch, CUDA graphs, VMM arenas) sees the
same limit -- a way to try a configuration sized for a smaller card on a B200.

    python -m xtier_b200.tools.vram_limit FREE_MIB WATCH_PID [--ready-file FILE]

--ready-file gets the MiB left free once the memory is held (a launch script waits for it).
(Reference parity: tools/vram_limit.py.)
"""
from __future__ import annotations

import argparse
import os
import sys
import time


def hold_bytes(free: int, free_mib: int) -> int:
    """Bytes to hold so that `free_mib` MiB stay free (<= 0: nothing to hold)."""
    return free - free_mib * (1 << 20)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('free_mib', type=int)
    ap.add_argument('watch_pid', type=int)
    ap.add_argument('--ready-file')
    a = ap.parse_args(argv)
    import torch
    free, total = torch.cuda.mem_get_info()
    hold = hold_bytes(free, a.free_mib)
    if hold <= 0:
        sys.exit(f'vram_limit: only {free >> 20} MiB free, nothing to hold for {a.free_mib} MiB')
    block = torch.empty(hold, dtype=torch.uint8, device='cuda')
    left, _ = torch.cuda.mem_get_info()
    print(f'vram_limit: holding {hold >> 20} MiB of {total >> 20} MiB; {left >> 20} MiB left for pid {a.watch_pid}',
          flush=True)
    if a.ready_file:
        with open(a.ready_file, 'w') as f:
            f.write(f'{left >> 20}\n')
    while os.path.exists(f'/proc/{a.watch_pid}'):
        time.sleep(1)
    del block
    return 0


if __name__ == '__main__':
    sys.exit(main())
