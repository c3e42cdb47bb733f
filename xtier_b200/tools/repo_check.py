"""Checks of this repository that need no GPU (the CPU test suite runs them). Exit status 1 on a finding.

- every Python file parses, every shell script passes `bash -n`, no file has Windows line ends;
- `xtier_b200/env_names.txt` is what the config registry generates, every XTIER_* name the sources, tests, run scripts
  and console cards mention is registered, and every registered name is used somewhere;
- every native function the Python side calls through ctypes (`xt_*` attributes of the loaded libraries) is defined
  with C linkage in csrc/, and every `extern "C"` function a header in csrc/include declares is defined.

    python -m xtier_b200.tools.repo_check
(Reference parity: tools/repo_check.py -- parse checks, the XTIER_* name list, native exports named by Python.)
"""
from __future__ import annotations

import ast
import re
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
NAME = re.compile(r'\bXTIER_[A-Z0-9_]*[A-Z0-9]\b')
PY_NATIVE = re.compile(r'\b(?:L|lib\(\)|_lib\(\)|self\._lib|lib)\.(xt_\w+)')
C_DEF = re.compile(r'^(?:extern\s+"C"\s+)?(?:[\w\*\s]+?)\b(xt_\w+)\s*\([^;]*?\)\s*\{', re.M | re.S)
C_DECL = re.compile(r'\b(xt_\w+)\s*\(')


def _files(*globs):
    out = []
    for g in globs:
        out += [p for p in ROOT.glob(g) if '_work' not in p.parts and '_build' not in p.parts
                and 'baseline' not in p.parts and 'gpurun_out' not in p.parts and '__pycache__' not in p.parts]
    return sorted(set(out))


def check_parse() -> list[str]:
    bad = []
    for p in _files('**/*.py'):
        try:
            ast.parse(p.read_text(encoding='utf-8'), str(p))
        except SyntaxError as e:
            bad.append(f'{p.relative_to(ROOT)}: {e}')
    bash = shutil.which('bash')
    for p in _files('**/*.sh'):
        if bash and subprocess.run([bash, '-n', str(p)], capture_output=True).returncode != 0:
            bad.append(f'{p.relative_to(ROOT)}: bash -n fails')
    for p in _files('**/*.py', '**/*.sh', '**/*.cpp', '**/*.cu', '**/*.cuh', '**/*.h', '**/*.md', '**/*.txt'):
        if b'\r\n' in p.read_bytes():
            bad.append(f'{p.relative_to(ROOT)}: Windows line ends')
    return bad


def check_names() -> list[str]:
    from .. import config
    bad = []
    listed = (ROOT / 'xtier_b200' / 'env_names.txt').read_text()
    if listed != config.env_names_text():
        bad.append('xtier_b200/env_names.txt differs from the registry (regenerate it from config.env_names_text())')
    registered = set(config.names())
    used = set()
    for p in _files('xtier_b200/**/*.py', 'csrc/**/*.cpp', 'csrc/**/*.cu', 'csrc/**/*.h', 'csrc/**/*.cuh',
                    'tests/*.py', 'bench.py', '__graft_entry__.py', 'configs/**/*'):
        if p.is_file() and p.name != 'env_names.txt':
            text = p.read_text(encoding='utf-8', errors='ignore')
            found = set(NAME.findall(text))
            if re.search(r"get\(['\"]XTIER['\"]\)", text):   # the master switch has no suffix
                found.add('XTIER')
            used |= found
            for n in sorted(found - registered):
                bad.append(f'{p.relative_to(ROOT)}: {n} is not registered in xtier_b200/config.py')
    for n in sorted(registered - used):
        bad.append(f'{n}: registered but used nowhere')
    return bad


def check_native() -> list[str]:
    bad = []
    defined = set()
    for p in _files('csrc/**/*.cpp', 'csrc/**/*.cu', 'csrc/**/*.h', 'csrc/**/*.cuh'):
        defined |= set(C_DEF.findall(p.read_text(encoding='utf-8', errors='ignore')))
    for p in _files('xtier_b200/**/*.py', 'tests/*.py', 'bench.py'):
        for n in sorted(set(PY_NATIVE.findall(p.read_text(encoding='utf-8')))):
            if n not in defined:
                bad.append(f'{p.relative_to(ROOT)}: calls {n}, which no csrc/ file defines')
    for p in _files('csrc/include/*.h'):
        for n in sorted(set(C_DECL.findall(p.read_text(encoding='utf-8')))):
            if n not in defined:
                bad.append(f'{p.relative_to(ROOT)}: declares {n}, which no csrc/ file defines')
    return bad


def run() -> list[str]:
    return check_parse() + check_names() + check_native()


def main(argv=None):
    found = run()
    for f in found:
        print(f)
    print('REPO-CHECK ' + ('FAIL' if found else 'PASS'), f'({len(found)} findings)' if found else '')
    return 1 if found else 0


if __name__ == '__main__':
    sys.exit(main())
