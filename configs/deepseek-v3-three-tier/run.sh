#!/usr/bin/env bash
# benchmark config 5 on one B200: DeepSeek-V3 shape at 32K context, each MoE layer's experts in three tiers -- GPU
# slots sized by the planner's auto-layout (20 % of the node's experts), the CPU engine's RAM (50 %), records on NVMe
# read on demand (30 %) -- plus a 4M x 4096 hashed-bigram table on NVMe looked up inside the decode graph.
# COLD_DIR and TABLE_DIR must be on a disk with room for the records and the 32 GiB table; LAYERS scales every tier.
set -euo pipefail
cd "$(dirname "$0")/../.."
exec python -m xtier_b200.tools.three_tier --layers "${LAYERS:-6}" --context "${CONTEXT:-32768}" \
    --cold-dir "${COLD_DIR:-/tmp/xtier-cold}" --table-dir "${TABLE_DIR:-/tmp/xtier-table}" \
    --table-rows "${TABLE_ROWS:-4194304}" "$@"
