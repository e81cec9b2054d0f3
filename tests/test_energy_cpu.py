"""Energy accounting (gateddeltanet_b200/energy.py) against a fake NVML on the CPU."""
import pytest

from gateddeltanet_b200 import energy


class FakeNVML:
    """Counter in mJ and power in mW; the counter can be made unsupported."""

    def __init__(self, counter=True, watts=500.0):
        self.counter = counter
        self.watts = watts
        self.mj = 1_000_000
        self.calls = []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlDeviceGetHandleByIndex(self, i):
        self.calls.append(("handle", i))
        return object()

    def nvmlDeviceGetTotalEnergyConsumption(self, h):
        if not self.counter:
            raise RuntimeError("not supported")
        self.mj += 250  # 0.25 J per query
        return self.mj

    def nvmlDeviceGetPowerUsage(self, h):
        return int(self.watts * 1000)


def test_counter_window_and_summary():
    nv = FakeNVML()
    m = energy.EnergyMeter(3, nvml=nv, sample_s=0.01)
    m.start()
    w = m.stop()
    assert w["method"] == "energy_counter"
    assert w["joules"] == pytest.approx(0.25)
    s = energy.summarize({"joules": 10.0, "seconds": 2.0, "method": "energy_counter"}, tokens=1000, idle_w=1.0)
    assert s["gross_j_per_token"] == pytest.approx(0.01)
    assert s["net_j_per_token"] == pytest.approx((10.0 - 2.0) / 1000)
    assert s["avg_power_w"] == pytest.approx(5.0)
    # only read-only queries were made
    assert all(c == "init" or c[0] == "handle" for c in nv.calls)


def test_trapezoid_fallback_and_nonpositive_net():
    nv = FakeNVML(counter=False, watts=400.0)
    m = energy.EnergyMeter(0, nvml=nv, sample_s=0.005)
    m.start()
    import time
    time.sleep(0.05)
    w = m.stop()
    assert w["method"] == "power_trapezoid"
    assert w["joules"] == pytest.approx(400.0 * w["seconds"], rel=0.05)
    s = energy.summarize(w, tokens=10, idle_w=1e6)
    assert s["net_j_per_token"] is None and s["net_tokens_per_j"] is None


def test_trapezoid_integral():
    assert energy.trapezoid([(0.0, 100.0), (1.0, 300.0), (3.0, 300.0)]) == pytest.approx(200.0 + 600.0)


def test_counter_going_backwards_is_an_error():
    nv = FakeNVML()
    m = energy.EnergyMeter(0, nvml=nv)
    m.start()
    nv.mj -= 10_000
    with pytest.raises(RuntimeError):
        m.stop()
