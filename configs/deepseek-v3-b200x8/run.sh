#!/usr/bin/env bash
# DeepSeek-V3 shape (benchmark config 3's model) served from one B200: HOT of each MoE layer's 256 experts in HBM
# slots, the rest on the CPU engine through the mailbox; random-init weights. With EP=N, the layer benchmark over N
# GPUs instead. Override any XTIER_* setting from the environment.
set -euo pipefail
cd "$(dirname "$0")/../.."
if [[ -n "${EP:-}" ]]; then
    exec timeout -k 60 1800 python -m torch.distributed.run --nnodes=1 --nproc-per-node "$EP" \
        --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29551}" -m xtier_b200.tools.ep_bench "$@"
fi
exec python -m xtier_b200.serve --model deepseek-v3 --hot "${HOT:-0.44}" --port "${PORT:-18190}" "$@"
