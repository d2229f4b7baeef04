"""Cost-model fitting and the calibration payload consumed by the planner configuration."""

import json

import numpy as np
import pytest

from placemoe_b200.placemoe.perf_model import LinkFit, PerfModel, fit_linear, robust_time


def test_fit_recovers_alpha_beta():
    sizes = [1e6, 4e6, 16e6, 64e6]
    times = [0.01 + 1.3e-9 * s for s in sizes]
    fit = fit_linear(sizes, times)
    assert abs(fit.alpha_ms - 0.01) < 1e-9 and abs(fit.beta_ms_per_byte - 1.3e-9) < 1e-15
    assert fit.r2 > 0.999999
    assert abs(fit.bandwidth_gbs - 1e-6 / 1.3e-9) < 1e-3


def test_fit_clamps_negative_latency_and_needs_two_sizes():
    fit = fit_linear([1.0, 2.0], [0.5, 1.5])  # alpha would be -0.5
    assert fit.alpha_ms == 0.0 and fit.beta_ms_per_byte > 0
    with pytest.raises(ValueError):
        fit_linear([3.0, 3.0], [1.0, 2.0])


def test_robust_time_is_median_of_rank_max():
    # ranks x repeats
    assert robust_time([[1.0, 5.0, 2.0], [2.0, 1.0, 3.0]]) == 3.0


def test_calibration_payload_is_accepted_by_runtime_config(tmp_path):
    from placemoe_b200.placemoe.runtime.config import PlaceMoECalibration

    m = PerfModel(links={"nvlink": LinkFit(0.01, 1.4e-9)}, compute=LinkFit(0.02, 3e-6), ranks_per_node=8, ep_size=8)
    assert m.select_dimension() == "direct"
    est = m.exchange_estimate([1e6, 2e6], [2e6, 1e6], assignments=[100, 200])
    assert est["comm_ms"] == pytest.approx(0.01 + 1.4e-9 * 2e6)
    assert est["compute_ms"] == pytest.approx(0.02 + 3e-6 * 200)
    path = tmp_path / "cal.json"
    m.save(str(path), scope={"ep_size": 8})
    cal = PlaceMoECalibration.from_mapping({"artifact": str(path)}, base_directory=tmp_path)
    c = cal.coefficients()
    assert c["intra_ms_per_byte"] == pytest.approx(1.4e-9)
    assert c["compute_ms_per_assignment"] == pytest.approx(3e-6)
    back = PerfModel.from_dict(json.loads(path.read_text())["fits"])
    assert back.links["nvlink"].beta_ms_per_byte == pytest.approx(1.4e-9)
    assert np.isfinite(back.links["nvlink"].bandwidth_gbs)
