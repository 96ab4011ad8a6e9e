"""Distributed runtime: process groups, sharded data parallelism, the
symmetric peer-memory data plane and the fused compute+collective kernels."""
