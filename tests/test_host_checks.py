"""Read-only host checks on a fake NVML and a fake cgroup tree: ownership reports exclude this
process, refusal covers busy and unanswerable GPUs, and cgroup counter deltas are computed and
reset-checked."""
from types import SimpleNamespace

import pytest

from qwen38_b200.utils.host_checks import OwnershipError, gpu_owners, host_snapshot, host_summary, preflight


class FakeNvml:
    def __init__(self, procs):
        self.procs = procs                    # {gpu: [(pid, bytes)]}, or an exception to raise

    def nvmlDeviceGetHandleByIndex(self, i):
        if i not in self.procs:
            raise RuntimeError("no such device")
        return i

    def nvmlDeviceGetComputeRunningProcesses(self, h):
        return [SimpleNamespace(pid=p, usedGpuMemory=b) for p, b in self.procs[h]]


def test_owners_exclude_self_and_report_memory():
    nv = FakeNvml({0: [(100, 3 << 30), (200, 1 << 20)], 1: [(100, 5 << 30)]})
    own = gpu_owners([0, 1, 2], nvml=nv, self_pid=100)
    assert own == {0: [{"pid": 200, "used_mib": 1}], 1: [], 2: None}


def test_preflight_refuses_busy_or_unknown_gpus():
    nv = FakeNvml({0: [(7, 1 << 30)], 1: []})
    rep = preflight([1], nvml=nv, self_pid=1)
    assert rep["busy"] == [] and rep["unknown"] == []
    assert preflight([0, 1], nvml=nv, self_pid=1)["busy"] == [0]
    with pytest.raises(OwnershipError):
        preflight([0], refuse=True, nvml=nv, self_pid=1)
    with pytest.raises(OwnershipError):
        preflight([3], refuse=True, nvml=nv, self_pid=1)        # NVML cannot answer for GPU 3
    assert preflight([0], nvml=None, self_pid=1)["unknown"] == [0]


def test_host_summary_deltas(tmp_path):
    (tmp_path / "cpu.stat").write_text("usage_usec 1000\nthrottled_usec 10\nnr_periods 5\n")
    (tmp_path / "memory.events").write_text("low 0\nhigh 1\noom 0\n")
    before = host_snapshot(tmp_path)
    assert "memory.pressure" in before["unavailable"]
    (tmp_path / "cpu.stat").write_text("usage_usec 4000\nthrottled_usec 2010\nnr_periods 9\n")
    (tmp_path / "memory.events").write_text("low 0\nhigh 3\noom 0\n")
    after = host_snapshot(tmp_path)
    s = host_summary(before, after)
    assert s["counter_deltas"]["cpu.stat"] == {"usage_usec": 3000, "throttled_usec": 2000, "nr_periods": 4}
    assert s["counter_deltas"]["memory.events"]["high"] == 2 and s["cpu_throttled_ms"] == 2.0
    (tmp_path / "cpu.stat").write_text("usage_usec 5\nthrottled_usec 0\nnr_periods 0\n")
    with pytest.raises(ValueError):
        host_summary(after, host_snapshot(tmp_path))
    with pytest.raises(ValueError):
        host_summary(after, before)
