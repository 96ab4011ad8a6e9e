"""Kernel value model: schedule features, 3-head surrogate + pairwise ranker."""
