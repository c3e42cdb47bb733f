"""The CPU engine library must run on AVX2-only hosts: AVX-512 instructions may appear only inside the functions the
source compiles for AVX-512 (`XT_AVX512` in csrc/engine/kernels.cpp), and 256-bit AVX only inside those and the
`XT_AVX2` ones. An inline helper (a std:: function, a lambda) that the compiler emits once, in the copy of an
AVX-512 function, and then calls from generic code would fault with SIGILL on such a host; this check finds it.

    python -m xtier_b200.tools.isa_check [--lib xtier_b200/_lib/libxt_engine.so]

Disassembles the built library (x86-64 code built here from this repository's sources) with objdump, assigns each
instruction to its function symbol, and compares against the function names the source marks. Also requires the
AVX-512 kernels to contain such instructions (otherwise the pattern would prove nothing). Exit status 1 on a finding.
(Reference parity: tools/isa_check.sh -- the same question for the reference's one-library-per-ISA build.)
"""
from __future__ import annotations

import argparse
import re
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
# zmm and mask registers, the EVEX-only xmm16-31 / ymm16-31, EVEX-only mnemonics
AVX512 = re.compile(r'zmm|%k[0-7]|%[xy]mm(1[6-9]|2[0-9]|3[01])\b|^\s*(vpternlog|vperm[it]2|vpcompress|vpexpand|'
                    r'vcompressp|vexpandp|vdpbf16|vcvtne2?ps2bf16|vfixupimm|vrndscale|vgetexp|vgetmant|vscalef|'
                    r'vrcp14|vrsqrt14|vpmullq|vpro[lr][dq]|vpsraq|vpabsq|vpm(ax|in)[su]q|vpermb|vpmultishiftqb|'
                    r'k(mov|and|or|xor|test|shift|not|unpck))')
YMM = re.compile(r'%ymm')
DECL = re.compile(r'^\s*(?:template\s*<[^>]*>\s*)?(XT_AVX512|XT_AVX2)\b[^(]*?\b(\w+)\s*\(', re.M)


def marked(source: str) -> dict[str, str]:
    """Function name -> 'avx512' / 'avx2' for the functions the source compiles for those targets."""
    return {m.group(2): m.group(1)[3:].lower() for m in DECL.finditer(source)}


def _base(symbol: str) -> str:
    """Plain function name of a (demangled) symbol: 'xt::dot_avx512_n<8, true>(...)' -> 'dot_avx512_n'."""
    s = symbol.split('(')[0]
    s = re.sub(r'<.*>$', '', s)
    s = s.split('::')[-1]
    return re.sub(r'\.(constprop|isra|part|cold|lto_priv)\.\d+.*$', '', s)


def scan(lib: str) -> dict[str, dict[str, int]]:
    """Per function symbol: counts of AVX-512 and 256-bit instructions."""
    out = subprocess.run(['objdump', '-d', '-C', '--no-show-raw-insn', lib], check=True, capture_output=True,
                         text=True).stdout
    fns: dict[str, dict[str, int]] = {}
    cur = None
    head = re.compile(r'^[0-9a-f]+ <(.+)>:$')
    for line in out.splitlines():
        m = head.match(line)
        if m:
            cur = m.group(1)
            continue
        if cur is None or '\t' not in line:
            continue
        ins = line.split('\t', 1)[1]
        ins = re.sub(r'<[^>]*>', '', ins)
        c = fns.setdefault(cur, {'avx512': 0, 'ymm': 0})
        if AVX512.search(ins):
            c['avx512'] += 1
        elif YMM.search(ins):
            c['ymm'] += 1
    return fns


def check(lib: str, source: str) -> list[str]:
    marks = marked(source)
    if not marks:
        return ['no XT_AVX512 / XT_AVX2 functions found in the source']
    findings = []
    fns = scan(lib)
    seen512 = 0
    for sym, c in fns.items():
        kind = marks.get(_base(sym))
        if c['avx512'] and kind != 'avx512':
            findings.append(f'{sym}: {c["avx512"]} AVX-512 instructions outside an XT_AVX512 function')
        if c['ymm'] and kind is None:
            findings.append(f'{sym}: {c["ymm"]} 256-bit AVX instructions outside an XT_AVX2 / XT_AVX512 function')
        if kind == 'avx512':
            seen512 += c['avx512']
    if seen512 == 0:
        findings.append('the XT_AVX512 functions contain no AVX-512 instructions: the check proves nothing')
    return findings


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--lib', default=str(ROOT / 'xtier_b200' / '_lib' / 'libxt_engine.so'))
    ap.add_argument('--source', default=str(ROOT / 'csrc' / 'engine' / 'kernels.cpp'))
    a = ap.parse_args(argv)
    found = check(a.lib, Path(a.source).read_text())
    for f in found:
        print(f)
    print('ISA-CHECK ' + ('FAIL' if found else 'PASS'))
    return 1 if found else 0


if __name__ == '__main__':
    sys.exit(main())
