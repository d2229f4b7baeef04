"""CPU tests of the PlaceMoE runtime control: strict config, scheduler, controller, planner command, CPU affinity."""

import json
import os

import pytest

from placemoe_b200.placemoe.runtime import (
    HotUpdateController,
    HotUpdateJob,
    HotUpdateScheduler,
    PlaceMoECalibration,
    PlaceMoEConfigurationError,
    PlaceMoEPlannerResources,
    PlaceMoERuntimeConfig,
    PlannerCommandSpec,
    UpdateKind,
    build_planner_command,
    discover_physical_cores,
    format_cpu_list,
    parse_cpu_list,
    planner_environment,
    resolve_cpu_affinity,
)


def write(p, text):
    p.write_text(text)
    return p


def test_config_paths_resolve_relative_to_yaml(tmp_path):
    (tmp_path / "sub").mkdir()
    cfg = write(tmp_path / "sub" / "pm.yaml", """
placemoe:
  initial_artifact: layout.json
  hot_update:
    enabled: true
    layout_interval_steps: 100
    mapping_interval_steps: 20
    work_root: work
  resources:
    workers: 4
""")
    c = PlaceMoERuntimeConfig.from_file(cfg)
    assert c.initial_artifact == str((tmp_path / "sub" / "layout.json").resolve())
    assert c.hot_update.work_root == str((tmp_path / "sub" / "work").resolve())
    assert c.hot_update.layout_interval_steps == 100 and c.resources.workers == 4


def test_config_rejects_unknown_and_bad_values(tmp_path):
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(write(tmp_path / "a.yaml", "bogus: 1\n"))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(write(tmp_path / "b.yaml", "hot_update: {failure_policy: maybe}\n"))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(write(tmp_path / "c.yaml", "hot_update: {enabled: true}\n"))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(write(tmp_path / "d.yaml", "resources: {planner_cpu_ids: '0-3'}\n"))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(write(tmp_path / "e.yaml", "calibration: {intra_ms_per_byte: -1}\n"))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoERuntimeConfig.from_file(tmp_path / "missing.yaml")


def test_calibration_artifact_and_scope(tmp_path):
    art = write(tmp_path / "cal.json", json.dumps({"status": "accepted", "scope": {"ep": 8, "hw": "b200"},
                                                   "coefficients": {"intra_ms_per_byte": 1e-9}}))
    c = PlaceMoECalibration.from_mapping({"artifact": "cal.json", "require_scope": True,
                                          "expected_scope": {"ep": 8, "hw": "b200"}}, base_directory=tmp_path)
    assert c.intra_ms_per_byte == 1e-9 and c.artifact == str(art.resolve())
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoECalibration.from_mapping({"artifact": "cal.json", "require_scope": True,
                                          "expected_scope": {"ep": 16}}, base_directory=tmp_path)
    write(tmp_path / "rej.json", json.dumps({"status": "rejected"}))
    with pytest.raises(PlaceMoEConfigurationError):
        PlaceMoECalibration.from_mapping({"artifact": "rej.json"}, base_directory=tmp_path)
    # explicit values override the artifact
    c2 = PlaceMoECalibration.from_mapping({"artifact": "cal.json", "intra_ms_per_byte": 2e-9}, base_directory=tmp_path)
    assert c2.intra_ms_per_byte == 2e-9


def test_environment_lookup(tmp_path):
    cfg = write(tmp_path / "x.json", json.dumps({"resources": {"workers": 2}}))
    assert PlaceMoERuntimeConfig.from_environment({"VEOMNI_PLACEMOE_CONFIG": str(cfg)}).resources.workers == 2
    assert PlaceMoERuntimeConfig.from_environment({}).initial_artifact == ""


def test_scheduler_coalesces_and_prefers_full():
    s = HotUpdateScheduler(layout_interval_steps=100, mapping_interval_steps=20, last_update_step=250)
    s.observe_step(20)
    s.observe_step(40)
    assert s.pop_next() is UpdateKind.MAPPING_ONLY and s.pop_next() is None
    s.observe_step(80)
    s.observe_step(100)  # full subsumes pending mapping
    assert s.pop_next() is UpdateKind.FULL and s.pop_next() is None
    s.observe_step(260)  # outside the window
    s.observe_step(0)
    assert s.pop_next() is None


def _job(kind=UpdateKind.FULL):
    return HotUpdateJob(kind, 1, (0,), 0.0, 0.0, "/tmp/j", "/tmp/j/l.json", "/tmp/j/r.json", "/tmp/j/log")


def test_controller_single_active_job_keeps_pending():
    c = HotUpdateController(layout_interval_steps=10, mapping_interval_steps=5, last_update_step=100)
    c.observe_step(5)
    assert c.next_update() is UpdateKind.MAPPING_ONLY
    c.start(_job(UpdateKind.MAPPING_ONLY))
    c.observe_step(10)
    assert c.next_update() is None  # job active: event stays pending
    with pytest.raises(RuntimeError):
        c.start(_job())
    assert c.finish() is not None
    assert c.next_update() is UpdateKind.FULL
    with pytest.raises(ValueError):
        HotUpdateController(1, 1, 1, failure_policy="ignore")


def test_planner_command_and_environment():
    spec = PlannerCommandSpec(python="py", planner_path="plan.py", route_root="/r", kind=UpdateKind.MAPPING_ONLY,
                              layer_keys=["a", "b"], ep_size=8, ranks_per_node=8, num_experts=128, slots_per_rank=20,
                              primary_slots_per_rank=16, redundant_slots_per_rank=4, hidden_size=2048,
                              bytes_per_element=2, output_layout="/o.json", output_report="/r.json",
                              input_layout="/in.json")
    res = PlaceMoEPlannerResources(workers=3, planner_cpu_ids="0-1", training_cpu_ids="2-7")
    cmd = build_planner_command(spec, PlaceMoECalibration(), res)
    assert cmd[:3] == ["taskset", "-c", "0-1"]
    assert cmd[cmd.index("--update-mode") + 1] == "mapping" and cmd[cmd.index("--input-layout") + 1] == "/in.json"
    assert cmd[cmd.index("--active-redundant-slots") + 1] == "32"
    with pytest.raises(ValueError):
        build_planner_command(PlannerCommandSpec(**{**spec.__dict__, "input_layout": ""}), PlaceMoECalibration(),
                              PlaceMoEPlannerResources())
    env = planner_environment(PlaceMoEPlannerResources(worker_threads=2), {})
    assert env["OMP_NUM_THREADS"] == "2" and env["MKL_NUM_THREADS"] == "2"


def _fake_sysfs(root, layout):
    """layout: list of (cpu, core, package, node)."""
    cpu_dir = root / "cpu"
    cpu_dir.mkdir(parents=True)
    (cpu_dir / "online").write_text(format_cpu_list([c for c, *_ in layout]))
    for cpu, core, pkg, node in layout:
        d = cpu_dir / f"cpu{cpu}"
        (d / "topology").mkdir(parents=True)
        (d / "topology" / "core_id").write_text(str(core))
        (d / "topology" / "physical_package_id").write_text(str(pkg))
        (d / f"node{node}").mkdir()
    return str(cpu_dir)


def test_cpu_affinity_numa_balanced_with_smt(tmp_path):
    # 2 NUMA nodes x 4 cores x 2 SMT threads = 16 cpus
    layout = []
    for node in range(2):
        for core in range(4):
            base = node * 4 + core
            layout.append((base, core, node, node))
            layout.append((base + 8, core, node, node))
    cores = discover_physical_cores(_fake_sysfs(tmp_path, layout))
    assert len(cores) == 8 and all(len(c.cpus) == 2 for c in cores)
    plan = resolve_cpu_affinity(cores)
    planner = parse_cpu_list(plan.planner_cpu_ids)
    training = parse_cpu_list(plan.training_cpu_ids)
    assert plan.planner_cores == 2 and len(planner) == 4
    assert not set(planner) & set(training) and len(planner) + len(training) == 16
    assert {c // 4 % 2 for c in planner if c < 8} | {(c - 8) // 4 for c in planner if c >= 8} == {0, 1}


def test_cpu_list_roundtrip():
    assert format_cpu_list([0, 1, 2, 5, 7, 8]) == "0-2,5,7-8"
    assert parse_cpu_list("0-2,5,7-8") == [0, 1, 2, 5, 7, 8]
    assert os.cpu_count() >= 1
