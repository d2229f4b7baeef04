"""CPU reservation for the planner process.

Physical cores are discovered from sysfs (``/sys/devices/system/cpu``): each
online CPU's core id, package id and NUMA node; SMT siblings form one core.
``resolve_cpu_affinity`` reserves at most 25 % of the physical cores for the
planner, spread evenly across NUMA nodes (highest-numbered cores of each
node), keeps SMT siblings together, and leaves the rest for training.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/runtime/cpu_affinity.py:14-262.
"""

from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class PhysicalCore:
    node: int
    package: int
    core: int
    cpus: tuple[int, ...]


@dataclass(frozen=True)
class CpuAffinityPlan:
    planner_cpu_ids: str
    training_cpu_ids: str
    planner_cores: int
    total_cores: int


def format_cpu_list(cpus) -> str:
    cpus = sorted(set(int(c) for c in cpus))
    if not cpus:
        return ""
    out, start, prev = [], cpus[0], cpus[0]
    for c in cpus[1:] + [None]:
        if c is not None and c == prev + 1:
            prev = c
            continue
        out.append(f"{start}-{prev}" if prev > start else f"{start}")
        if c is not None:
            start = prev = c
    return ",".join(out)


def parse_cpu_list(text: str) -> list[int]:
    out = []
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            out.extend(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return sorted(set(out))


def _read(path: str) -> str | None:
    try:
        with open(path) as f:
            return f.read().strip()
    except OSError:
        return None


def discover_physical_cores(sysfs_root: str = "/sys/devices/system/cpu", allowed: set[int] | None = None
                            ) -> list[PhysicalCore]:
    online = _read(os.path.join(sysfs_root, "online"))
    cpus = parse_cpu_list(online) if online else []
    if allowed is not None:
        cpus = [c for c in cpus if c in allowed]
    groups: dict[tuple[int, int, int], list[int]] = {}
    for c in cpus:
        base = os.path.join(sysfs_root, f"cpu{c}")
        core = _read(os.path.join(base, "topology", "core_id"))
        pkg = _read(os.path.join(base, "topology", "physical_package_id"))
        node = 0
        try:
            for entry in os.listdir(base):
                if entry.startswith("node") and entry[4:].isdigit():
                    node = int(entry[4:])
                    break
        except OSError:
            pass
        key = (node, int(pkg) if pkg else 0, int(core) if core else c)
        groups.setdefault(key, []).append(c)
    return [PhysicalCore(k[0], k[1], k[2], tuple(sorted(v))) for k, v in sorted(groups.items())]


def resolve_cpu_affinity(cores: list[PhysicalCore] | None = None, *, fraction: float = 0.25,
                         max_planner_cores: int | None = None) -> CpuAffinityPlan:
    if cores is None:
        allowed = set(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None
        cores = discover_physical_cores(allowed=allowed)
    total = len(cores)
    if total < 2:
        cpus = [c for core in cores for c in core.cpus]
        return CpuAffinityPlan("", format_cpu_list(cpus), 0, total)
    want = max(1, int(total * fraction))
    if max_planner_cores is not None:
        want = min(want, max_planner_cores)
    want = min(want, total - 1)
    by_node: dict[int, list[PhysicalCore]] = {}
    for core in cores:
        by_node.setdefault(core.node, []).append(core)
    nodes = sorted(by_node)
    picked: list[PhysicalCore] = []
    i = 0
    while len(picked) < want:
        node = nodes[i % len(nodes)]
        pool = [c for c in by_node[node] if c not in picked]
        if pool:
            picked.append(pool[-1])
        i += 1
        if i > 4 * total:
            break
    planner = [c for core in picked for c in core.cpus]
    training = [c for core in cores if core not in picked for c in core.cpus]
    return CpuAffinityPlan(format_cpu_list(planner), format_cpu_list(training), len(picked), total)


def apply_training_affinity(plan: CpuAffinityPlan) -> bool:
    if not plan.training_cpu_ids or not hasattr(os, "sched_setaffinity"):
        return False
    os.sched_setaffinity(0, parse_cpu_list(plan.training_cpu_ids))
    return True
