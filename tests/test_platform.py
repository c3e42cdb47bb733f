"""Host-side serving fixes on the CPU: page-cache advice on checkpoint files (and through SafeTensors.close), and the
frozen GC heap."""
import gc

import numpy as np
import torch

from xtier_b200.utils import platform


def test_file_cache_advice(tmp_path):
    files = []
    for i in range(3):
        f = tmp_path / f'f{i}.bin'
        f.write_bytes(np.random.default_rng(i).bytes(1 << 20))
        files.append(f)
    assert platform.read_ahead(files[0])
    assert platform.drop_file_cache(files + [tmp_path / 'missing']) == 3


def test_safetensors_close_drops_the_pages_it_mapped(tmp_path, monkeypatch):
    from xtier_b200.models import hf
    path = tmp_path / 'm.safetensors'
    hf.save_safetensors(path, {'a': torch.arange(12, dtype=torch.float32).view(3, 4)})
    st = hf.SafeTensors(path)
    dropped = []
    monkeypatch.setattr(platform, 'drop_file_cache', lambda paths: dropped.append(list(paths)) or len(paths))
    assert st.get('a')[2, 3].item() == 11.0
    st.close()
    assert dropped == [[str(path)]]
    st2 = hf.SafeTensors(path)
    st2.close()                    # nothing mapped: nothing to drop
    assert len(dropped) == 1


def test_freeze_gc():
    try:
        n = platform.freeze_gc()
        assert n > 0 and gc.get_freeze_count() == n
    finally:
        gc.unfreeze()
