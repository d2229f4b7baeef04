"""materialize_config writes a configuration that validate_config and the runtime loader accept."""

import json

from placemoe_b200.placemoe import materialize_config, validate_config
from placemoe_b200.placemoe.runtime.config import PlaceMoERuntimeConfig


def test_materialize_then_validate(tmp_path):
    out = tmp_path / "run" / "placemoe.yaml"
    info = materialize_config.materialize(str(out), ep_size=4, num_experts=16, layers=3, redundant=1,
                                          seed="eplb", hot_update=True, layout_interval=50, mapping_interval=10)
    assert info["topology"]["slots_per_rank"] == 5
    cfg = PlaceMoERuntimeConfig.from_file(str(out))
    assert cfg.hot_update.enabled and cfg.hot_update.mapping_interval_steps == 10
    rep = validate_config.validate(str(out), ep_size=4, num_experts=16, slots_per_rank=5, layers=3)
    assert rep["errors"] == [], rep
    assert rep["artifact"]["layers"] == 3
    bad = validate_config.validate(str(out), ep_size=8)
    assert any("ep_size" in e for e in bad["errors"])


def test_validate_reports_schema_errors(tmp_path):
    p = tmp_path / "bad.yaml"
    p.write_text("placemoe:\n  hot_update:\n    enabled: true\n    bogus_key: 3\n")
    rep = validate_config.validate(str(p))
    assert rep["errors"] and "config" in rep["errors"][0]
    assert validate_config.main([str(p)]) == 1
    json.dumps(rep)
