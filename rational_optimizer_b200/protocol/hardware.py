"""GPU selection and exclusivity audit for one NVSwitch node.

The published protocol picked four A6000s forming two NVLink pairs
(reference experiments/protocol/select_nvlink_gpus.py:86-105,
audit_runtime_hardware.py).  On an HGX B200 node every GPU reaches every
other through NVSwitch, so the requirement becomes: the selected GPUs are
all of the expected model, pairwise NVLink-connected (``NV<k>`` in
``nvidia-smi topo -m``), idle (no compute process, little memory used) and
unthrottled.  Reads go through an injectable NVML-like object so the logic
is tested on CPU against a fake; nothing here changes any GPU setting.
"""
from __future__ import annotations

import argparse
import itertools
import json
import re
import subprocess
import sys

EXPECTED_GPU_NAME = "NVIDIA B200"
# clock-event reason bits that disqualify a timing run (NVML constants)
THROTTLE_BITS = {"hw_slowdown": 0x08, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                 "hw_power_brake_slowdown": 0x80}


def normalize_uuid(value) -> str:
    if value is None:
        return ""
    if isinstance(value, bytes):
        value = value.decode()
    text = str(value).strip()
    if text and not text.upper().startswith("GPU-") and re.fullmatch(
            r"[0-9A-Fa-f]{8}-[0-9A-Fa-f]{4}-[0-9A-Fa-f]{4}-[0-9A-Fa-f]{4}-[0-9A-Fa-f]{12}", text):
        text = f"GPU-{text}"
    return text.upper()


def topology_peer_values(topology: str) -> dict:
    """``{row GPU index: {column GPU index: link token}}`` from ``nvidia-smi topo -m``."""
    rows = {}
    for line in topology.splitlines():
        fields = line.split()
        if not fields or re.fullmatch(r"GPU[0-9]+", fields[0]) is None or "X" not in fields[1:]:
            continue
        rows[fields[0][3:]] = fields[1:]
    cols = sorted(rows, key=int)
    return {r: dict(zip(cols, vals)) for r, vals in rows.items()}


def nvlink_edges(topology: str, indices) -> list:
    peers = topology_peer_values(topology)
    sel = [str(i) for i in indices]
    return [(a, b) for i, a in enumerate(sel) for b in sel[i + 1:]
            if peers.get(a, {}).get(b, "").startswith("NV")]


def fully_connected(topology: str, indices) -> bool:
    n = len(list(indices))
    return len(nvlink_edges(topology, indices)) == n * (n - 1) // 2


class SmiNvml:
    """Minimal NVML-like reader backed by the ``nvidia_ml_py`` bindings."""

    def __init__(self):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()

    def count(self):
        return self.nv.nvmlDeviceGetCount()

    def info(self, i):
        h = self.nv.nvmlDeviceGetHandleByIndex(i)
        name = self.nv.nvmlDeviceGetName(h)
        mem = self.nv.nvmlDeviceGetMemoryInfo(h)
        procs = self.nv.nvmlDeviceGetComputeRunningProcesses(h)
        reasons = self.nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        return {"index": i, "uuid": self.nv.nvmlDeviceGetUUID(h),
                "name": name.decode() if isinstance(name, bytes) else name,
                "memory_used_mib": mem.used // (1 << 20), "processes": len(procs), "clock_reasons": int(reasons)}


def topology_text() -> str:
    return subprocess.run(["nvidia-smi", "topo", "-m"], check=True, text=True, capture_output=True,
                          timeout=60).stdout


def audit(nvml, topology: str, indices, *, expected_name=EXPECTED_GPU_NAME, max_memory_mib=1024) -> dict:
    """Return an audit record; ``passed`` is False with ``problems`` listed otherwise."""
    problems, devices = [], []
    for i in indices:
        d = nvml.info(int(i))
        devices.append(d)
        if expected_name and expected_name not in d["name"]:
            problems.append(f"GPU {i} is {d['name']!r}, expected {expected_name!r}")
        if d["processes"]:
            problems.append(f"GPU {i} runs {d['processes']} other compute process(es)")
        if d["memory_used_mib"] > max_memory_mib:
            problems.append(f"GPU {i} has {d['memory_used_mib']} MiB in use")
        bad = [k for k, bit in THROTTLE_BITS.items() if d["clock_reasons"] & bit]
        if bad:
            problems.append(f"GPU {i} clock events active: {bad}")
    if len(list(indices)) > 1 and not fully_connected(topology, indices):
        problems.append("selected GPUs are not pairwise NVLink-connected")
    return {"schema": "rational_optimizer_b200_hardware_audit_v1", "indices": [int(i) for i in indices],
            "devices": devices, "passed": not problems, "problems": problems}


def select(nvml, topology: str, count: int, **kw) -> dict:
    """Lowest-numbered ``count`` GPUs that pass :func:`audit` together."""
    healthy = [i for i in range(nvml.count()) if audit(nvml, topology, [i], **kw)["passed"]]
    for combo in itertools.combinations(healthy, count):
        rec = audit(nvml, topology, combo, **kw)
        if rec["passed"]:
            rec["cuda_visible_devices"] = ",".join(str(i) for i in combo)
            return rec
    raise RuntimeError(f"no {count} idle, pairwise NVLink-connected {kw.get('expected_name', EXPECTED_GPU_NAME)} GPUs")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--count", type=int, default=8)
    ap.add_argument("--expected-name", default=EXPECTED_GPU_NAME)
    ap.add_argument("--max-memory-mib", type=int, default=1024)
    a = ap.parse_args(argv)
    rec = select(SmiNvml(), topology_text(), a.count, expected_name=a.expected_name,
                 max_memory_mib=a.max_memory_mib)
    print(json.dumps(rec, sort_keys=True))
    return 0


if __name__ == "__main__":
    sys.exit(main())
