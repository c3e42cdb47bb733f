#!/usr/bin/env bash
# Qwen3-style MoE (benchmark config 2) on one B200: 40% of each layer's experts in GPU hot slots, the rest on the CPU
# engine through the mailbox. Override any XTIER_* setting from the environment.
set -euo pipefail
cd "$(dirname "$0")/../.."
export XTIER_CACHE_ADAPT=${XTIER_CACHE_ADAPT:-1}
exec python -m xtier_b200.serve --model qwen3-moe --hot "${HOT:-0.4}" --port "${PORT:-18180}" "$@"
