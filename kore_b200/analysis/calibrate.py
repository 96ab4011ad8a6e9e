"""Peak calibration on the local GPU: a STREAM-style copy (HBM bytes/s) and a
large square bf16 matmul (FLOP/s), timed with CUDA events after warm-up,
written as a MEASURED_PEAKS.json-style dict that the rooflines read.
Reference parity: kore/analysis/calibrate_peaks.py:58-117 (STREAM triad +
square-matmul calibration)."""
from __future__ import annotations

import argparse
import json

import torch


def measure(n_bytes: int = 4 << 30, mm: int = 8192, iters: int = 20) -> dict:
    from ..bench.timing import median_ms, time_cuda
    a = torch.empty(n_bytes // 2, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    copy_ms = median_ms(time_cuda(lambda: b.copy_(a), iters, flush_l2=False))
    x = torch.randn(mm, mm, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(mm, mm, device="cuda", dtype=torch.bfloat16)
    mm_ms = median_ms(time_cuda(lambda: x @ y, iters, flush_l2=False))
    return {"hbm_gbs": 2 * n_bytes / copy_ms / 1e6, "bf16_tflops": 2 * mm ** 3 / mm_ms / 1e9,
            "device": torch.cuda.get_device_name(), "source": "kore_b200.analysis.calibrate"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore calibrate")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    r = measure()
    print(json.dumps(r))
    if a.out:
        json.dump(r, open(a.out, "w"), indent=2)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
