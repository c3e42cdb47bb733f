"""Web console: pick a model card (configs/*/console.py), set its options, launch / stop its server, follow its log and
health. Stdlib only (reference parity: xtier/console)."""
