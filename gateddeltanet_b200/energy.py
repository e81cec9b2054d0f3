"""GPU energy per decoded token from NVML (read-only queries).

Follows the reference's GPU energy protocol (c_impl/doc/gpu_latency_energy_
evaluation.md sec. 5; scripts/run_gpu_power_eval.py): gross energy is the
difference of NVML's total-energy counter (millijoules) across the active
window; where the counter is unsupported or does not advance, the sampled
power trace is integrated with trapezoids. A counter that goes backwards is an
error. Idle power is measured over a loaded-idle window (the process alive,
no decode), and the idle-subtracted energy per token is null when the net
energy is not positive.

Nothing here changes a GPU setting: only nvmlInit, handle lookup, the energy
counter and the power reading are used. The NVML module is injectable so the
arithmetic is tested on the CPU against a fake.
"""
from __future__ import annotations

import threading
import time
from typing import Optional


class EnergyMeter:
    def __init__(self, index: int, nvml=None, sample_s: float = 0.05):
        if nvml is None:
            import pynvml as nvml  # noqa: N813
        self.nvml = nvml
        self.nvml.nvmlInit()
        self.handle = self.nvml.nvmlDeviceGetHandleByIndex(index)
        self.sample_s = sample_s
        self._samples: list[tuple[float, float]] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._e0: Optional[int] = None
        self._t0 = 0.0

    def _counter(self) -> Optional[int]:
        try:
            return int(self.nvml.nvmlDeviceGetTotalEnergyConsumption(self.handle))
        except Exception:
            return None

    def _power_w(self) -> Optional[float]:
        try:
            return self.nvml.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
        except Exception:
            return None

    def _sampler(self):
        while not self._stop.is_set():
            p = self._power_w()
            if p is not None:
                self._samples.append((time.perf_counter(), p))
            self._stop.wait(self.sample_s)

    def start(self) -> None:
        self._samples = []
        self._stop.clear()
        self._e0 = self._counter()
        self._t0 = time.perf_counter()
        p = self._power_w()
        if p is not None:
            self._samples.append((self._t0, p))
        self._thread = threading.Thread(target=self._sampler, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        """Gross joules and seconds of the window since start(), and the method used."""
        e1 = self._counter()
        t1 = time.perf_counter()
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)
        p = self._power_w()
        if p is not None:
            self._samples.append((t1, p))
        seconds = t1 - self._t0
        if self._e0 is not None and e1 is not None:
            if e1 < self._e0:
                raise RuntimeError("NVML energy counter went backwards")
            if e1 > self._e0:
                return {"joules": (e1 - self._e0) / 1000.0, "seconds": seconds, "method": "energy_counter",
                        "samples": len(self._samples)}
        return {"joules": trapezoid(self._samples), "seconds": seconds, "method": "power_trapezoid",
                "samples": len(self._samples)}

    def idle_watts(self, seconds: float = 1.0) -> float:
        """Mean power over a loaded-idle window of `seconds`."""
        self.start()
        time.sleep(seconds)
        w = self.stop()
        return w["joules"] / w["seconds"] if w["seconds"] > 0 else 0.0


def trapezoid(samples: list[tuple[float, float]]) -> float:
    """Integral of (time, watts) samples in joules."""
    e = 0.0
    for (t0, p0), (t1, p1) in zip(samples, samples[1:]):
        e += 0.5 * (p0 + p1) * (t1 - t0)
    return e


def summarize(window: dict, tokens: int, idle_w: Optional[float]) -> dict:
    """J/token and tokens/J, gross and idle-subtracted (null when the net energy is not positive)."""
    j, s = window["joules"], window["seconds"]
    out = {"joules": round(j, 4), "seconds": round(s, 4), "tokens": tokens, "method": window["method"],
           "avg_power_w": round(j / s, 2) if s > 0 else None,
           "gross_j_per_token": round(j / tokens, 6) if tokens else None,
           "gross_tokens_per_j": round(tokens / j, 3) if j > 0 else None,
           "idle_power_w": round(idle_w, 2) if idle_w is not None else None}
    net = None if idle_w is None else j - idle_w * s
    if net is not None and net > 0 and tokens:
        out["net_j_per_token"] = round(net / tokens, 6)
        out["net_tokens_per_j"] = round(tokens / net, 3)
    else:
        out["net_j_per_token"] = None
        out["net_tokens_per_j"] = None
    return out
