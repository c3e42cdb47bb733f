"""Parallel encoding of long prompts: with a byte-level BPE fast tokenizer (trained here on this repository's
sources) the sliced batch encoding gives exactly the ids of encoding the whole text, also around added tokens that
contain a newline."""
from pathlib import Path

import pytest

from xtier_b200.utils.tokenize import parallel_encode, supported

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope='module')
def tok():
    tokenizers = pytest.importorskip('tokenizers')
    transformers = pytest.importorskip('transformers')
    from tokenizers import decoders, models, pre_tokenizers, trainers
    files = [str(p) for p in sorted((ROOT / 'xtier_b200').rglob('*.py'))[:40]]
    t = tokenizers.Tokenizer(models.BPE())
    t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    t.decoder = decoders.ByteLevel()
    t.train(files, trainers.BpeTrainer(vocab_size=2000, special_tokens=['<|endoftext|>'], show_progress=False))
    fast = transformers.PreTrainedTokenizerFast(tokenizer_object=t)
    fast.add_special_tokens({'additional_special_tokens': ['<|im_start|>', '<|im_end|>\n']})
    return fast


def test_parallel_encode_is_exact(tok):
    assert supported(tok)
    text = '\n'.join(p.read_text() for p in sorted((ROOT / 'xtier_b200').rglob('*.py')))
    text += '<|im_start|>user\nHello<|im_end|>\nAnd more text\n' * 50
    want = tok(text, add_special_tokens=False)['input_ids']
    got = parallel_encode(tok, text, target_chars=4096)
    assert got == want and len(got) > 10000
    short = 'x = 1\n'
    assert parallel_encode(tok, short) == tok(short, add_special_tokens=False)['input_ids']
