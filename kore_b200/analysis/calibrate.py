"""Peak calibration on the local GPU: a STREAM-style copy (HBM bytes/s) and a
large square bf16 matmul (FLOP/s), timed with CUDA events after warm-up, both
as a burst (median of short runs) and, for the matmul, sustained (back to back
for ``sustain_s`` seconds, where a 1 kW part settles under its power cap),
with the SM clock and power sampled read-only through NVML meanwhile;
written as a MEASURED_PEAKS.json-style dict that the rooflines read.
Reference parity: kore/analysis/calibrate_peaks.py:58-117 (STREAM triad +
square-matmul calibration)."""
from __future__ import annotations

import argparse
import json

import torch


def measure(n_bytes: int = 4 << 30, mm: int = 8192, iters: int = 20, sustain_s: float = 0.0) -> dict:
    from ..bench.timing import median_ms, time_cuda
    a = torch.empty(n_bytes // 2, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    copy_ms = median_ms(time_cuda(lambda: b.copy_(a), iters, flush_l2=False))
    x = torch.randn(mm, mm, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(mm, mm, device="cuda", dtype=torch.bfloat16)
    mm_ms = median_ms(time_cuda(lambda: x @ y, iters, flush_l2=False))
    out = {"hbm_gbs": 2 * n_bytes / copy_ms / 1e6, "bf16_tflops": 2 * mm ** 3 / mm_ms / 1e9,
           "device": torch.cuda.get_device_name(), "source": "kore_b200.analysis.calibrate"}
    if sustain_s > 0:
        samples = _NvmlSampler()
        samples.start()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(1, int(sustain_s * 1e3 / max(mm_ms, 1e-3)))
        e0.record()
        for _ in range(n):
            x @ y
        e1.record()
        torch.cuda.synchronize()
        samples.stop()
        out["bf16_tflops_sustained"] = 2 * mm ** 3 * n / e0.elapsed_time(e1) / 1e9
        out["clocks_under_load"] = samples.summary()
    return out


class _NvmlSampler:
    """SM clock and power every 200 ms on a thread (read-only NVML queries)."""

    def __init__(self, index: int = 0):
        import threading
        self.index, self.mhz, self.watts = index, [], []
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - no NVML: no clock record
            return

        def run():
            while not self._stop.is_set():
                try:
                    self.mhz.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    self.watts.append(pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0)
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        m = sorted(self.mhz)
        return {"samples": len(m), "sm_mhz_median": m[len(m) // 2] if m else None, "sm_max_mhz": self.max_mhz,
                "power_w_max": max(self.watts) if self.watts else None}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore calibrate")
    ap.add_argument("--out", default="")
    ap.add_argument("--sustain-s", type=float, default=4.0, help="seconds of back-to-back GEMMs (0: burst only)")
    a = ap.parse_args(argv)
    r = measure(sustain_s=a.sustain_s)
    print(json.dumps(r))
    if a.out:
        json.dump(r, open(a.out, "w"), indent=2)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
