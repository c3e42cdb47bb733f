"""Command-line tools: python -m xtier_b200.tools.<name> (plan_probe, plan_trace, plan_auto, plan_calibrate,
cold_relayout)."""
