"""In-tree native build (no JIT cache): the libraries land in xtier_b200/_lib/ and travel with the source tree.

  libxt_engine.so  CPU expert engine + cold-expert store (C++17, per-function ISA targets)     csrc/engine, csrc/cold
  libxt_rows.so    NVMe row tables (C++17)                                                    csrc/tables
  libxt_cuda.so    sm_100a kernels, the CPU<->GPU mailbox host side and the torch op bindings  csrc/cuda, csrc/mailbox

Every CUDA source is compiled with `-gencode arch=compute_100a,code=sm_100a` (B200 only; tcgen05/TMA need the `a`
variant). The .cu files include no torch headers, so they compile in seconds; one binding file registers the ops with
TORCH_LIBRARY, and the library is loaded with torch.ops.load_library (no pybind, no JIT). Rebuilds are incremental by
modification time of each object's source and of every header under csrc/.

    python -m xtier_b200._build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / 'csrc'
LIB = Path(__file__).resolve().parent / '_lib'
OBJ = ROOT / '_build'
CUDA_HOME = Path(os.environ.get('CUDA_HOME', '/usr/local/cuda'))
NVCC = str(CUDA_HOME / 'bin' / 'nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
CXXFLAGS = ['-O3', '-std=c++17', '-fPIC', '-pthread', '-g1', '-Wall', '-Wno-unused-function', '-Wno-sign-compare']


def _cutlass_include() -> list[str]:
    """CuTe/CUTLASS headers vendored in the image (used as source by the tcgen05 kernels)."""
    for cand in (Path(sysconfig.get_paths()['purelib']) / 'flashinfer' / 'data' / 'cutlass' / 'include',):
        if (cand / 'cute').is_dir():
            return [f'-I{cand}']
    return []


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce
    inc = [f'-I{p}' for p in ce.include_paths(device_type='cuda')]
    libdir = Path(torch.__file__).parent / 'lib'
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f'-D_GLIBCXX_USE_CXX11_ABI={abi}', '-DTORCH_API_INCLUDE_EXTENSION_H', '-DTORCH_EXTENSION_NAME=xt_cuda']
    libs = [f'-L{libdir}', '-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu', '-ltorch_cuda', f'-Wl,-rpath,{libdir}']
    return inc, defs, libs


def _headers_mtime() -> float:
    m = 0.0
    for p in CSRC.rglob('*'):
        if p.suffix in ('.h', '.cuh', '.hpp', '.inl'):
            m = max(m, p.stat().st_mtime)
    return m


def _stale(out: Path, srcs: list[Path], extra_mtime: float = 0.0) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs) or extra_mtime > t


def _run(cmd: list[str]):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'build failed: {" ".join(cmd)}\n{r.stdout}\n{r.stderr}')
    return r


def _compile(src: Path, force: bool, hdr: float, extra: list[str]) -> Path:
    obj = OBJ / (src.relative_to(CSRC).as_posix().replace('/', '__') + '.o')
    if force or _stale(obj, [src], hdr):
        obj.parent.mkdir(parents=True, exist_ok=True)
        if src.suffix == '.cu':
            cmd = [NVCC, *ARCH, '-O3', '-lineinfo', '-std=c++17', '--expt-relaxed-constexpr', '-Xcompiler',
                   '-fPIC', '-Xptxas=-v' if os.environ.get('XT_PTXAS_V') else '-w', '-c', str(src), '-o', str(obj),
                   f'-I{CSRC}', *_cutlass_include(), *extra]
        else:
            cmd = ['g++', *CXXFLAGS, '-c', str(src), '-o', str(obj), f'-I{CSRC}', f'-I{CUDA_HOME / "include"}', *extra]
        _run(cmd)
    return obj


def _link(out: Path, objs: list[Path], libs: list[str], force: bool):
    if force or _stale(out, objs):
        tmp = out.with_suffix('.so.tmp')
        _run(['g++', '-shared', '-o', str(tmp), *map(str, objs), *libs])
        os.replace(tmp, out)   # atomic: a running process keeps its mapping of the old file


def build(force: bool = False, jobs: int | None = None, cuda: bool = True, verbose: bool = True):
    LIB.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    jobs = jobs or max(2, os.cpu_count() or 2)
    with cf.ThreadPoolExecutor(jobs) as ex:
        eng = [ex.submit(_compile, s, force, hdr, []) for s in
               (CSRC / 'engine' / 'engine.cpp', CSRC / 'engine' / 'kernels.cpp', CSRC / 'cold' / 'store.cpp')]
        rows = [ex.submit(_compile, CSRC / 'tables' / 'rows.cpp', force, hdr, [])] \
            if (CSRC / 'tables' / 'rows.cpp').exists() else []
        cu_objs = []
        if cuda:
            inc, defs, tlibs = _torch_flags()
            cu_srcs = sorted((CSRC / 'cuda').glob('*.cu')) + sorted((CSRC / 'mailbox').glob('*.cu'))
            host_srcs = sorted((CSRC / 'mailbox').glob('*.cpp'))
            bind_srcs = sorted((CSRC / 'cuda').glob('*.cpp'))
            cu_objs = [ex.submit(_compile, s, force, hdr, []) for s in cu_srcs]
            cu_objs += [ex.submit(_compile, s, force, hdr, []) for s in host_srcs]
            cu_objs += [ex.submit(_compile, s, force, hdr, [*inc, *defs]) for s in bind_srcs]
        eng_o = [f.result() for f in eng]
        _link(LIB / 'libxt_engine.so', eng_o, ['-pthread'], force)
        if rows:
            _link(LIB / 'libxt_rows.so', [f.result() for f in rows], ['-pthread'], force)
        if cuda:
            objs = [f.result() for f in cu_objs]
            libs = [*tlibs, f'-L{CUDA_HOME / "lib64"}', '-lcudart_static', '-lrt', '-ldl', '-pthread',
                    f'-L{LIB}', '-lxt_engine', '-Wl,-rpath,$ORIGIN']
            _link(LIB / 'libxt_cuda.so', objs, libs, force)
    if verbose:
        print('xtier_b200: native build ok:', ', '.join(sorted(p.name for p in LIB.glob('*.so'))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('-j', type=int, default=None)
    ap.add_argument('--no-cuda', action='store_true')
    a = ap.parse_args()
    build(force=a.force, jobs=a.j, cuda=not a.no_cuda)


if __name__ == '__main__':
    main()
