"""Roofline models, arch peaks and bottleneck analysis for sm_100a."""
