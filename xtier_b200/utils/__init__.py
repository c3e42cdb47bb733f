"""Small shared helpers (serving metrics)."""
