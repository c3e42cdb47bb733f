"""XTIER_* settings: one declarative registry, read from the environment.

Every switch is declared once below (name, kind, default, one line of help). `get(name)` parses it, `names()` lists
them (the committed `env_names.txt` is generated from this table and checked by a test), and `check_environment()`
warns about XTIER_* variables nobody reads (a typo would otherwise silently do nothing). The public surface follows
the reference's switches (xtier/config.py:1-46, xtier/env_names.txt) where they mean the same thing here; settings
that only exist for SGLang or for the reference's SM120 packs are not carried over.
"""
from __future__ import annotations

import dataclasses
import logging
import os

logger = logging.getLogger('xtier_b200')


@dataclasses.dataclass(frozen=True)
class Setting:
    name: str
    kind: str          # 'flag' | 'int' | 'float' | 'str' | 'list' (cpu/layer list '0-3,8')
    default: object
    help: str


_S = Setting
SETTINGS: tuple[Setting, ...] = (
    _S('XTIER', 'flag', True, 'master switch of the tiered MoE layers (0: every expert on the GPU, no CPU tier)'),
    _S('XTIER_LAYERS', 'str', 'all', 'model layers whose routed experts are tiered: all or a list 0-11,20'),
    _S('XTIER_THREADS', 'int', 0, 'CPU expert engine workers (0: every CPU but one for the mailbox dispatcher)'),
    _S('XTIER_ISA', 'str', 'auto', 'CPU engine kernels: auto, avx512 (AVX-512 BF16), avx2, scalar'),
    _S('XTIER_L2_PREFETCH', 'int', 1, 'decode graphs prefetch the next layer\'s dense weights and KV cache into L2'),
    _S('XTIER_GEMM_PAIR', 'int', 0, '1: BF16 GEMMs with M >= 1024 run the CTA-pair (tcgen05 cta_group::2) kernel'),
    _S('XTIER_SPIN_US', 'int', 200, 'engine workers spin this long before sleeping on a futex'),
    _S('XTIER_MAIN_CPUS', 'str', '', 'CPUs of the other threads of the process (auto: all but the workers)'),
    _S('XTIER_DISPATCH_CPU', 'int', -1, 'CPU the mailbox dispatcher thread is pinned to (-1: last CPU)'),
    _S('XTIER_WORKER_CPUS', 'list', '', 'CPUs the engine workers are pinned to (empty: every allowed CPU; set by placement)'),
    _S('XTIER_PDL', 'flag', True, 'programmatic dependent launch between the decode kernels (0: plain stream order)'),
    _S('XTIER_ATTN_CUDA_CORES', 'flag', False, 'decode attention on the CUDA-core kernel for every group size'),
    _S('XTIER_DECODE_MAX', 'int', 64, 'calls of up to this many tokens use the mailbox decode path (graph capturable)'),
    _S('XTIER_SLOT_TOKENS', 'int', 16, 'tokens of one mailbox decode slot at the most'),
    _S('XTIER_CPU_TIMEOUT_S', 'float', 60.0, 'a mailbox request unanswered for this long fails the step (bounded wait)'),
    _S('XTIER_CACHE_SLOTS', 'int', -1, 'GPU hot-expert slots per layer (-1: every expert, 0: none)'),
    _S('XTIER_CACHE_FRACTION', 'float', 0.0, 'hot slots as a fraction of the experts (overrides CACHE_SLOTS when >0)'),
    _S('XTIER_CACHE_FULL', 'list', '', 'layers that keep every expert on the GPU'),
    _S('XTIER_CACHE_PLAN', 'str', '', 'planner output {"slots": {layer: n}} or "auto"'),
    _S('XTIER_CACHE_PROFILE', 'str', '', 'route-count profile that fills the hot slots at start'),
    _S('XTIER_CACHE_ADAPT', 'flag', True, 'adaptive hot-expert swaps from decayed route counts'),
    _S('XTIER_CACHE_EVERY', 'int', 4, 'decode windows between policy rounds'),
    _S('XTIER_CACHE_SWAPS', 'int', 16, 'swaps per policy round at most'),
    _S('XTIER_CACHE_DECAY', 'float', 0.7, 'decay of the route counts per round'),
    _S('XTIER_CACHE_MIN_GAIN', 'float', 1.5, 'minimum count advantage of an incoming expert over its victim'),
    _S('XTIER_CACHE_LOG', 'int', 0, 'log the cache statistics every N policy rounds (0: off)'),
    _S('XTIER_DECODE_MISS_GPU', 'float', 0.0, 'share of a token\'s CPU-tier routes the GPU computes from pinned host '
       'memory over PCIe (one per token at most; 0: off)'),
    _S('XTIER_GC_FREEZE', 'flag', True, 'the server freezes the Python heap once the model is built (no GC scans of '
       'the model\'s objects while serving)'),
    _S('XTIER_EP_PCIE_SLOTS', 'int', -1, 'expert parallelism with a RAM CPU tier: GPU staging slots for CPU-tier '
       'experts the GPU reads from the engine\'s host memory over PCIe while the engine computes the others (0: off, '
       '-1: XTIER_EP_PCIE_SHARE of the CPU-tier experts a call is expected to touch)'),
    _S('XTIER_EP_PCIE_SHARE', 'float', 0.37, 'share of the touched CPU-tier experts read over PCIe when '
       'XTIER_EP_PCIE_SLOTS is -1 (the balance of ~0.5 ms per expert over PCIe against ~0.3 ms on 14 engine threads; '
       'planner.cost.staging_share of probed coefficients gives it for another machine)'),
    _S('XTIER_CACHE_RING', 'flag', True, 'hot-slot swaps copy on a side stream and the decode step maps them'),
    _S('XTIER_CACHE_ELASTIC', 'flag', False, 'extra hot slots in VMM-backed memory that prefills take back'),
    _S('XTIER_CACHE_ELASTIC_MAX', 'float', 2.0, 'address space per layer, as a multiple of its base hot slots'),
    _S('XTIER_CACHE_ELASTIC_RESERVE_GIB', 'float', 2.0, 'free device memory never given to extra slots'),
    _S('XTIER_CACHE_ELASTIC_CRITICAL_GIB', 'float', 1.0, 'free memory under this releases every extra slot'),
    _S('XTIER_CACHE_ELASTIC_MARGIN', 'float', 1.25, 'factor on the predicted need of an allocating forward'),
    _S('XTIER_CACHE_ELASTIC_IDLE', 'int', 32, 'decode steps after an allocating forward before slots grow again'),
    _S('XTIER_CACHE_ELASTIC_CHECK', 'int', 16, 'decode steps between critical-memory checks'),
    _S('XTIER_CACHE_ELASTIC_COOLDOWN_S', 'float', 600.0, 'no growth for this long after a critical release'),
    _S('XTIER_CACHE_ELASTIC_EXTRAPOLATE', 'float', 2.0, 'how far a learnt need is scaled up to bound a larger one'),
    _S('XTIER_GPU2_SLOTS', 'str', '', 'auto / on: the hot slots of all GPUs of the process group form one pool, '
       'read over NVLink'),
    _S('XTIER_EP', 'int', 0, 'expert-parallel ranks of the hot-slot pool (0: the world size)'),
    _S('XTIER_EP_ORDER', 'int', 1, 'EP expert streams take the routes grouped by expert slot (0: arrival order)'),
    _S('XTIER_COLD', 'flag', False, 'cold experts in NVMe relayout files, read on demand with O_DIRECT'),
    _S('XTIER_COLD_DIR', 'str', '', 'directories (one per drive, comma separated) of the cold-expert store'),
    _S('XTIER_COLD_FRACTION', 'float', 0.0, 'share of each layer\'s experts kept cold (not in RAM)'),
    _S('XTIER_COLD_THREADS', 'int', 4, 'reader threads per cold-store file'),
    _S('XTIER_COLD_PARTS', 'str', '', 'cold records dealt over the drives by these weights, e.g. 5:5:2 (default equal)'),
    _S('XTIER_COLD_UNITS', 'int', 1, 'units per cold record (1: whole NUMA shards; 3: gate / up / rest dealt apart)'),
    _S('XTIER_COLD_HALF_LIFE', 'float', 50.0, 'half life (engine calls) of the use counts that pick cold victims'),
    _S('XTIER_FAST_LOAD', 'flag', False, 'read expert tensors straight from safetensors into engine shards (O_DIRECT)'),
    _S('XTIER_SPEC_TRUNCATE_Q', 'float', 0.2, 'speculative verify truncated after the first draft with q < this (0: off)'),
    _S('XTIER_SPEC_DRAFT_TEMP_SCALE', 'float', 0.8, 'a sampled request\'s draft runs at its temperature x this'),
    _S('XTIER_CKPT_FORMAT', 'str', 'nvfp4', 'expert format unquantized (BF16) checkpoints are quantized to: nvfp4 or mxfp4'),
    _S('XTIER_LOAD_DIGEST', 'flag', False, 'log a digest of every loaded layer'),
    _S('XTIER_TAIL_SKIP', 'str', '', 'K/N: decode calls of top-N skip experts outside every token\'s K largest routes'),
    _S('XTIER_TAIL_SKIP_TOKENS', 'int', 8, 'tail skip applies to calls of at most this many tokens'),
    _S('XTIER_GPU_PREFILL_MIN', 'int', 1024, 'prefill calls of at least this many tokens run every expert on the GPU'),
    _S('XTIER_HYBRID_PREFILL_MAX', 'int', 2560, 'partly cached prefill below this: GPU hot routes || CPU the rest'),
    _S('XTIER_PREFILL_CHUNK', 'int', 8, 'experts uploaded per chunk of the host-resident GPU prefill'),
    _S('XTIER_LONG_PREFILL_CHUNK', 'int', 0, 'tokens per chunk of a long prompt\'s prefill (0: one piece)'),
    _S('XTIER_PREFILL_SLOTS', 'int', 4, 'staging slots of the prefill upload ring'),
    _S('XTIER_ROUTE_TRACE', 'str', '', 'binary route trace of the CPU decode calls (planner input)'),
    _S('XTIER_TIMING', 'flag', False, 'log synchronized MoE time per forward'),
    _S('XTIER_PREFILL_PROFILE', 'flag', False, 'CUDA events per prefill phase'),
    _S('XTIER_PREFILL_MX', 'flag', False, 'grouped prefill of MXFP4 experts with MXFP8 activations (kind::mxf8f6f4)'),
    _S('XTIER_PREFILL_ATTN', 'str', 'tc', 'prefill attention: tc (this framework\'s tcgen05 kernel) or sdpa (PyTorch)'),
    _S('XTIER_ATTN_PREFILL_EMU', 'int', 0, 'prefill attention: exponential pairs of every 8 computed on the FMA pipe'),
    _S('XTIER_DEBUG_BOUNDS', 'flag', False, 'flash MLA checks every selected cache slot: an out-of-range one is skipped '
       'and sets the error word to 2'),
    _S('XTIER_DEBUG_STALL_US', 'int', 0, 'test only: the mailbox dispatcher stalls this long per request'),
    _S('XTIER_DEBUG_SEQ_START', 'int', 0, 'test only: first sequence number of the swap ring (wrap tests)'),
    _S('XTIER_ROWS_MODE', 'str', 'direct', 'row tables: direct (O_DIRECT reads) or ram (mapped and locked)'),
    _S('XTIER_ROWS_IO_THREADS', 'int', 32, 'row-table IO threads'),
    _S('XTIER_ROWS_CACHE_MB', 'int', 1024, 'row-table cache size'),
    _S('XTIER_PLAN_LAMBDA', 'float', 0.0, 'planner weight of the upload cost (0: sweep)'),
    _S('XTIER_PLANNER_PROBE', 'str', '', 'planner probe file (plan_probe output) for XTIER_CACHE_PLAN=auto'),
    _S('XTIER_PLANNER_TRACE', 'str', '', 'route profile for XTIER_CACHE_PLAN=auto'),
    _S('XTIER_CACHE_BUDGET_GIB', 'float', 0.0, 'GPU memory for hot slots over all layers (planner budget)'),
    _S('XTIER_ENGINE_LIB', 'str', '', 'path of the CPU engine library (default: the in-tree build)'),
    _S('XTIER_CONSOLE_PORT', 'int', 8765, 'console HTTP port'),
    _S('XTIER_PACKS', 'str', 'all', 'model packs: all, none or a list'),
)

_BY_NAME = {s.name: s for s in SETTINGS}


def cpulist(text: str) -> list[int]:
    """'0-3,8' -> [0, 1, 2, 3, 8]"""
    out: list[int] = []
    for part in str(text).replace(' ', '').replace('\n', '').split(','):
        if part:
            lo, _, hi = part.partition('-')
            out.extend(range(int(lo), int(hi or lo) + 1))
    return out


def _parse(s: Setting, raw: str):
    if s.kind == 'flag':
        return raw.strip().lower() in ('1', 'true', 'yes', 'on')
    if s.kind == 'int':
        return int(raw)
    if s.kind == 'float':
        return float(raw)
    if s.kind == 'list':
        return cpulist(raw)
    return raw


def get(name: str):
    s = _BY_NAME[name]
    raw = os.environ.get(name)
    if raw is None or raw.strip() == '':
        return cpulist(s.default) if s.kind == 'list' else s.default
    try:
        return _parse(s, raw)
    except ValueError as e:
        raise ValueError(f'xtier_b200: {name}={raw!r} is not a valid {s.kind}') from e


def names() -> list[str]:
    return sorted(_BY_NAME)


def unknown_names(environ=None) -> list[str]:
    env = os.environ if environ is None else environ
    return sorted(k for k in env if k.startswith('XTIER') and k not in _BY_NAME)


def check_environment(environ=None) -> list[str]:
    bad = unknown_names(environ)
    for k in bad:
        logger.warning('xtier_b200: %s is set but no setting of that name exists (typo?)', k)
    return bad


def layer_selected(layer: int) -> bool:
    spec = str(get('XTIER_LAYERS')).strip()
    return spec in ('', 'all') or layer in cpulist(spec)


def env_names_text() -> str:
    return '\n'.join(names()) + '\n'


def help_text() -> str:
    return '\n'.join(f'{s.name}={s.default!s:8} {s.help}' for s in sorted(SETTINGS, key=lambda s: s.name))
