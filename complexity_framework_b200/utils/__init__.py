"""Utilities: checkpointing, profiling, security, device policy."""
