"""tasks/train_text.py and tasks/train_vlm.py run end to end on CPU (tiny model, 2 steps)."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(task, tmp_path, extra=()):
    cfg = tmp_path / "cfg.yaml"
    cfg.write_text("model:\n  preset: tiny_qwen3_moe\ndata:\n  max_seq_len: 320\n")
    out = tmp_path / "out"
    cmd = [sys.executable, os.path.join(ROOT, "tasks", task), str(cfg), "--train.max_steps=2",
           "--train.global_batch_size=2", "--train.micro_batch_size=1", f"--train.output_dir={out}",
           "--train.log_interval=1", *extra]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="4")
    env.pop("VEOMNI_PLACEMOE_CONFIG", None)
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    return r, out


@pytest.mark.timeout(900)
def test_train_text_entrypoint(tmp_path):
    r, out = _run("train_text.py", tmp_path)
    assert "step 2/2" in r.stdout
    lines = [json.loads(x) for x in (out / "metrics.jsonl").read_text().splitlines()]
    assert lines and lines[-1]["step"] == 2 and lines[-1]["env/tokens_per_s"] > 0
    assert any(k.startswith("router/max_over_mean/") for k in lines[-1])
    assert (out / "veomni_cli.yaml").exists()


@pytest.mark.timeout(900)
def test_train_vlm_entrypoint(tmp_path):
    r, out = _run("train_vlm.py", tmp_path)
    assert "step 2/2" in r.stdout
