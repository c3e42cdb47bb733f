"""Host-side fixes for a serving process: page-cache eviction of checkpoint files once their tensors are loaded,
read-ahead of a file before its tensors are read, and a frozen garbage-collector heap once the model is built.

A checkpoint read through memory maps leaves its pages in the page cache (hundreds of GB for a large MoE), where they
compete with the CPU tier's expert memory and the pinned buffers; `drop_file_cache` tells the kernel they are not
needed again (posix_fadvise DONTNEED; clean pages go at once). `read_ahead` asks for a file's pages before the first
tensor of it is read (WILLNEED), so the disk streams while the previous file's tensors are converted. After the build,
the Python heap holds millions of long-lived objects (tensors, layer dicts); `freeze_gc` moves them to the permanent
generation so that collections during serving stop scanning them (no pauses of tens of milliseconds between tokens).

Reference parity: xtier/platform.py:169 (`_drop_file_cache`: checkpoint page-cache eviction plus read-ahead) and the
GC freeze of `install_serving` (:474); parallel BPE encoding is utils/tokenize.py. The SGLang-specific fixes of that
file (TileLang target, TP1 token-id all-reduce skip, SM120 MXFP8 tactic, JIT cache links, image decode) have no
counterpart in a standalone framework.
"""
from __future__ import annotations

import gc
import os


def _advise(path, advice) -> bool:
    try:
        fd = os.open(str(path), os.O_RDONLY)
    except OSError:
        return False
    try:
        os.posix_fadvise(fd, 0, 0, advice)
        return True
    except OSError:
        return False
    finally:
        os.close(fd)


def drop_file_cache(paths) -> int:
    """Evicts the clean page-cache pages of `paths`; returns how many files were advised."""
    return sum(_advise(p, os.POSIX_FADV_DONTNEED) for p in paths)


def read_ahead(path) -> bool:
    """Starts reading `path` into the page cache in the background."""
    return _advise(path, os.POSIX_FADV_WILLNEED)


def freeze_gc() -> int:
    """Collects once, then moves every live object to the permanent generation; returns the frozen object count."""
    gc.collect()
    gc.freeze()
    return gc.get_freeze_count()
