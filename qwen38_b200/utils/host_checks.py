"""Read-only host checks around a run: who else holds the GPUs, and what the host's cgroup counters
did during a request.

* ``gpu_owners`` / ``preflight``: the reference refuses to open its cards while another process
  holds them (``scripts/ci/device-owners.py``, a scan of /proc file descriptors).  On B200 the same
  question goes to NVML (compute processes per GPU, with their memory); ``preflight`` reports them
  and, when asked, refuses to start.  Nothing here changes a device setting or resets a GPU.
* ``host_snapshot`` / ``host_summary``: cgroup v2 CPU, memory and pressure counters before and after
  a request and their deltas (``scripts/ci/request_host_health.py``), to tell a slow run caused by
  host contention (throttled CPU time, memory pressure) from a slow device.

    python -m qwen38_b200.utils.host_checks --gpus 0 1      # owners report as JSON
"""
from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path


class OwnershipError(RuntimeError):
    pass


def _nvml():
    try:
        import pynvml
        pynvml.nvmlInit()
        return pynvml
    except Exception:
        return None


def gpu_owners(indices, nvml="auto", self_pid: int | None = None) -> dict:
    """{gpu index: [{"pid", "used_mib"}]} of compute processes other than ``self_pid`` (this
    process by default).  Returns None per GPU when NVML cannot answer."""
    nv = _nvml() if nvml == "auto" else nvml
    me = os.getpid() if self_pid is None else self_pid
    out = {}
    for i in indices:
        if nv is None:
            out[i] = None
            continue
        try:
            h = nv.nvmlDeviceGetHandleByIndex(i)
            procs = nv.nvmlDeviceGetComputeRunningProcesses(h)
        except Exception:
            out[i] = None
            continue
        rows = []
        for p in procs:
            if int(p.pid) == me:
                continue
            used = getattr(p, "usedGpuMemory", None)
            rows.append({"pid": int(p.pid), "used_mib": None if used is None else int(used) >> 20})
        out[i] = rows
    return out


def preflight(indices, *, refuse: bool = False, nvml="auto", self_pid: int | None = None) -> dict:
    """Ownership report for ``indices``; with ``refuse``, raises ``OwnershipError`` when another
    process holds one of them or NVML cannot prove them free."""
    owners = gpu_owners(indices, nvml=nvml, self_pid=self_pid)
    busy = {i: rows for i, rows in owners.items() if rows}
    unknown = [i for i, rows in owners.items() if rows is None]
    report = {"owners": owners, "busy": sorted(busy), "unknown": unknown,
              "scope": "snapshot of NVML compute processes; not a reservation"}
    if refuse and (busy or unknown):
        raise OwnershipError(f"GPUs not proven free: busy {sorted(busy)}, unknown {unknown}")
    return report


CGROUP_FILES = ("cpu.stat", "cpu.max", "cpu.pressure", "memory.current", "memory.peak", "memory.events",
                "memory.swap.current", "memory.pressure", "io.pressure")


def host_snapshot(root: str | Path = "/sys/fs/cgroup") -> dict:
    snap = {"monotonic_ns": time.monotonic_ns(), "cgroup": {}, "unavailable": {}}
    for name in CGROUP_FILES:
        try:
            snap["cgroup"][name] = (Path(root) / name).read_text().strip()
        except OSError as e:
            snap["unavailable"][name] = type(e).__name__
    return snap


def _counters(text: str) -> dict:
    out = {}
    for line in text.splitlines():
        parts = line.split()
        if len(parts) == 2 and parts[1].isdigit():
            out[parts[0]] = int(parts[1])
    return out


def host_summary(before: dict, after: dict) -> dict:
    """Elapsed time and the deltas of the monotonic cgroup counters (cpu.stat, memory.events)
    between two snapshots; raises if a counter went backwards (a reset makes them meaningless)."""
    elapsed = after["monotonic_ns"] - before["monotonic_ns"]
    if elapsed <= 0:
        raise ValueError("snapshots out of order")
    deltas = {}
    for name in ("cpu.stat", "memory.events"):
        if name in before["cgroup"] and name in after["cgroup"]:
            a, b = _counters(before["cgroup"][name]), _counters(after["cgroup"][name])
            deltas[name] = {k: b[k] - a[k] for k in a.keys() & b.keys()}
            if any(v < 0 for v in deltas[name].values()):
                raise ValueError(f"{name} counters went backwards between the snapshots")
    throttled = deltas.get("cpu.stat", {}).get("throttled_usec")
    return {"elapsed_ms": elapsed / 1e6, "counter_deltas": deltas, "cpu_throttled_ms": None if throttled is None
            else throttled / 1e3, "scope": "whole interval between the snapshots; not proof of exclusive host use"}


def main(argv=None):
    ap = argparse.ArgumentParser(description="read-only GPU ownership and host health report")
    ap.add_argument("--gpus", type=int, nargs="*", default=[0])
    ap.add_argument("--refuse", action="store_true", help="exit non-zero unless every GPU is proven free")
    a = ap.parse_args(argv)
    try:
        rep = preflight(a.gpus, refuse=a.refuse)
    except OwnershipError as e:
        print(json.dumps({"error": str(e)}))
        return 1
    rep["host"] = host_snapshot()
    print(json.dumps(rep, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
