"""The fixed-seed regression tool: a run compared with its own baseline passes; a perturbed tensor, a missing
tensor and a slower step fail with the documented thresholds."""

import json
import os

import torch

from verl_omni_b200.cli import regress as R


def test_second_run_matches_bootstrapped_baseline(tmp_path):
    args = ["--out", str(tmp_path), "--steps", "2", "--dump-steps", "1,2", "--perf-skip-steps", "1", "--no-perf",
            "--strict", "trainer.device=cpu"]
    assert R.main(args) == 2  # strict: no baseline yet
    args = args[:-2] + args[-1:]
    assert R.main(args) == 0  # creates the baseline
    base = tmp_path / "baseline" / "flowgrpo_tiny"
    p = torch.load(base / "step_1" / "payload.pt", weights_only=True)
    assert {"batch.latents", "batch.old_log_probs", "batch.advantages", "grad_norms"} <= set(p)
    assert R.main(args) == 0  # same seeds on CPU: bit-identical
    rep = json.load(open(tmp_path / "current" / "flowgrpo_tiny" / "dump_compare.json"))
    assert rep["ok"] and all(e["max_abs_err"] == 0.0 for e in rep["files"]["step_2"].values())


def _write(d, step, payload):
    os.makedirs(os.path.join(d, f"step_{step}"), exist_ok=True)
    torch.save(payload, os.path.join(d, f"step_{step}", "payload.pt"))


def test_precision_thresholds(tmp_path):
    x = torch.linspace(-1, 1, 1000)
    img = torch.rand(2, 3, 8, 8)
    _write(tmp_path / "b", 1, {"batch.log_probs": x, "batch.responses": img, "gone": x})
    _write(tmp_path / "c", 1, {"batch.log_probs": x + 5e-5, "batch.responses": img + 1.5 / 255})
    rep = R.compare_dumps(str(tmp_path / "c"), str(tmp_path / "b"))
    assert rep["files"]["step_1"]["batch.log_probs"]["ok"]  # 5e-5 < atol 1e-4
    assert rep["files"]["step_1"]["batch.responses"]["ok"]  # image tolerance 2/255
    assert not rep["ok"] and any("gone" in f for f in rep["failures"])
    _write(tmp_path / "c2", 1, {"batch.log_probs": x + 3e-4, "batch.responses": img, "gone": x})
    rep = R.compare_dumps(str(tmp_path / "c2"), str(tmp_path / "b"))
    assert not rep["ok"] and not rep["files"]["step_1"]["batch.log_probs"]["ok"]


def test_perf_thresholds():
    base = {"perf/time_per_step": 10.0, "timing_s/update_weights": 1.0, "perf/throughput": 5.0}
    ok = R.compare_metrics({"perf/time_per_step": 11.0, "timing_s/update_weights": 1.18, "perf/throughput": 4.5},
                           base)
    assert ok["ok"], ok
    bad = R.compare_metrics({"perf/time_per_step": 11.6, "timing_s/update_weights": 1.0, "perf/throughput": 5.0},
                            base)
    assert not bad["ok"] and "perf/time_per_step" in bad["failures"][0]
    bad = R.compare_metrics({"perf/time_per_step": 10.0, "timing_s/update_weights": 1.0, "perf/throughput": 4.0},
                            base)
    assert not bad["ok"]
    assert R.summarise([{"perf/time_per_step": 99.0}, {"perf/time_per_step": 2.0}, {"perf/time_per_step": 4.0}],
                       1)["perf/time_per_step"] == 3.0
