"""Communication / compute cost model for the planner, fitted on the machine.

Every transfer class is modelled as ``t(bytes) = alpha + beta * bytes`` (ms),
fitted by least squares on timed probes (median over repeats of the max over
ranks).  On one NVSwitch domain there is a single link class for expert
traffic (GPU to GPU over NVLink 5); the model keeps the reference's split
between "intra" and "inter" coefficients so that calibration files stay
interchangeable, and maps both to the NVLink fit unless a multi-node fit is
supplied.  Expert compute is fitted the same way per routed assignment.

``calibration_payload`` writes the reference's calibration JSON shape
(``status: accepted`` + six ``coefficients``) so the result plugs into
``VEOMNI_PLACEMOE_CONFIG.calibration.artifact`` unchanged.

Reference parity: veomni/distributed/moe/hiermoe/perf_model.py:31-90
(linear link fits), :91-229 (startup probe fitting), :229-328 (hierarchical
time estimate), :330-493 (dimension selection); topology.py:21-82.  On one
NVSwitch level the dimension selection always resolves to direct
(rank-level) dedup.
"""

from __future__ import annotations

import dataclasses
import json
import math
from typing import Iterable, Mapping, Sequence

import numpy as np


@dataclasses.dataclass(frozen=True)
class LinkFit:
    """t(ms) = alpha_ms + beta_ms_per_byte * bytes."""

    alpha_ms: float
    beta_ms_per_byte: float
    r2: float = 1.0
    samples: int = 0

    def time_ms(self, nbytes: float) -> float:
        return self.alpha_ms + self.beta_ms_per_byte * float(nbytes)

    @property
    def bandwidth_gbs(self) -> float:
        return 1e-6 / self.beta_ms_per_byte if self.beta_ms_per_byte > 0 else math.inf


def fit_linear(sizes: Sequence[float], times_ms: Sequence[float]) -> LinkFit:
    """Least-squares alpha + beta * size; alpha is clamped at 0 (a probe cannot be faster than free)."""
    x = np.asarray(sizes, dtype=np.float64)
    y = np.asarray(times_ms, dtype=np.float64)
    if x.size < 2 or np.ptp(x) == 0:
        raise ValueError("a linear fit needs at least two distinct sizes")
    A = np.stack([np.ones_like(x), x], 1)
    (alpha, beta), *_ = np.linalg.lstsq(A, y, rcond=None)
    if alpha < 0:
        alpha = 0.0
        beta = float((x @ y) / (x @ x))
    pred = alpha + beta * x
    ss_res = float(((y - pred) ** 2).sum())
    ss_tot = float(((y - y.mean()) ** 2).sum()) or 1.0
    return LinkFit(float(alpha), float(beta), 1.0 - ss_res / ss_tot, int(x.size))


def robust_time(samples_per_rank: Iterable[Sequence[float]]) -> float:
    """Median over repeats of the max over ranks (the reference's probe statistic)."""
    arr = np.asarray([list(s) for s in samples_per_rank], dtype=np.float64)  # [ranks, repeats]
    return float(np.median(arr.max(axis=0)))


@dataclasses.dataclass
class PerfModel:
    """Fitted link classes and compute rate for one EP group."""

    links: dict[str, LinkFit]
    compute: LinkFit | None = None  # t(ms) per routed assignment (alpha per layer call)
    ranks_per_node: int = 8
    ep_size: int = 8

    def a2a_ms(self, bytes_out_per_rank: float, link: str = "nvlink") -> float:
        return self.links[link].time_ms(bytes_out_per_rank)

    def exchange_estimate(self, send_bytes: Sequence[float], recv_bytes: Sequence[float],
                          assignments: Sequence[float] | None = None) -> dict[str, float]:
        """Time of one dispatch/combine exchange: the slowest rank's max(send, recv) over the link,
        plus (optionally) the slowest rank's expert compute."""
        link = self.links.get("nvlink") or next(iter(self.links.values()))
        comm = max(link.time_ms(max(s, r)) for s, r in zip(send_bytes, recv_bytes))
        comp = 0.0
        if assignments is not None and self.compute is not None:
            comp = max(self.compute.time_ms(a) for a in assignments)
        return {"comm_ms": comm, "compute_ms": comp, "total_ms": comm + comp}

    def select_dimension(self) -> str:
        """Dedup hierarchy: one NVSwitch domain has no node level, so always rank-level ("direct")."""
        return "direct" if self.ep_size <= self.ranks_per_node else "hierarchical"

    # ---------------------------------------------------------------- I/O
    def to_dict(self) -> dict:
        return {"ranks_per_node": self.ranks_per_node, "ep_size": self.ep_size,
                "links": {k: dataclasses.asdict(v) for k, v in self.links.items()},
                "compute": dataclasses.asdict(self.compute) if self.compute else None}

    @classmethod
    def from_dict(cls, d: Mapping) -> "PerfModel":
        return cls(links={k: LinkFit(**v) for k, v in d["links"].items()},
                   compute=LinkFit(**d["compute"]) if d.get("compute") else None,
                   ranks_per_node=int(d.get("ranks_per_node", 8)), ep_size=int(d.get("ep_size", 8)))

    def calibration_payload(self, scope: Mapping | None = None, base: Mapping[str, float] | None = None) -> dict:
        """Planner calibration JSON (reference format).  Fitted coefficients replace the
        per-byte link costs and the per-assignment compute cost; the others come from
        ``base`` (default: the runtime configuration's defaults)."""
        from .runtime.config import DEFAULT_COEFFICIENTS

        link = self.links.get("nvlink") or next(iter(self.links.values()))
        inter = self.links.get("inter", link)
        coeffs = dict(base or DEFAULT_COEFFICIENTS)
        coeffs["inter_ms_per_byte"] = inter.beta_ms_per_byte
        coeffs["intra_ms_per_byte"] = link.beta_ms_per_byte
        if self.compute is not None:
            coeffs["compute_ms_per_assignment"] = self.compute.beta_ms_per_byte
        return {"status": "accepted", "scope": dict(scope or {}), "coefficients": coeffs,
                "fits": self.to_dict()}

    def save(self, path: str, scope: Mapping | None = None) -> None:
        with open(path, "w") as f:
            json.dump(self.calibration_payload(scope), f, indent=2)
