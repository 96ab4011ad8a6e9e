"""Micro-benchmarks of the native kernels (CUDA-event timed, L2 flushed)."""
