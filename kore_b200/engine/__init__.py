"""Execution engines: the explicit forward/backward training engine, the
rollout (generation) engine and their shared step helpers."""
