"""Acceptance tools against a running `xtier_b200.serve` (stdlib HTTP client; prompts from a tokenizer and a corpus,
or seeded ids for a random-init model):

    speed.py        decode speed (streamed, per request and aggregate), prefill latency by prompt length, long-context
                    prefill + decode
    quality.py      fixed-text perplexity with top-N dumps, the KL lower bound between two dumps, token stability across
                    recomputed prompts
    copy_test.py    verbatim copy of source windows (a real instruction-tuned checkpoint)
    agent.py        coding-agent sessions over the chat API with sandboxed tools, sized to target contexts
    robustness.py   aborted streams, refused requests, concurrent requests; a long prompt beside a decoding request

`bench.py` at the repository root is the driver's throughput benchmark; these measure a served model as a client sees
it. (Reference parity: bench/*.py of the reference, which drive an SGLang server the same way.)
"""
