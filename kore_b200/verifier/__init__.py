"""Hardware-counter collection (Nsight Compute) and compiler-report parsing."""
