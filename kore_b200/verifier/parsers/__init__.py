"""Parsers for Nsight Compute CSV exports and ptxas / nvcc reports."""
from .ncu import KernelCounters, parse_ncu_long_csv, parse_ncu_raw_csv  # noqa: F401
from .ptxas import RegisterInfo, parse_nvcc_diagnostics, parse_ptxas_report  # noqa: F401
