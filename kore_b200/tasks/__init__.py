"""Kernel tasks: operator library, task ABI, registry with held-out split,
and the subprocess driver contract of the verifier."""
