"""Fixed-seed precision and performance regression check of a FlowGRPO run.

    python -m verl_omni_b200.cli.regress --out OUT [--case NAME] [--steps 6] [--dump-steps 1,2]
        [--perf-skip-steps 2] [--strict] [trainer overrides ...]

Runs ``--steps`` training steps of the configured trainer (defaults: the tiny DiT on this machine's device)
and writes ``OUT/current/<case>/``:

* ``step_<k>/payload.pt`` for every step in ``--dump-steps``: the step's batch tensors after the actor update
  (``batch.<key>``: rollout latents, timesteps, rollout / old log-probs, advantages, scores, decoded images
  when kept, ...) and the gradient seen by the optimizer step (``gradients.<param>`` in full for adapter
  parameters, ``grad_norms`` -- one L2 norm per trainable parameter -- for full fine-tunes);
* ``metrics.jsonl`` (every step's metrics) and ``metrics.json`` (the mean of each compared metric over the
  steps after ``--perf-skip-steps``);
* ``dump_compare.json`` / ``metrics_compare.json`` against ``OUT/baseline/<case>/`` and the exit status.

A missing baseline is created from the current run unless ``--strict`` is given (then it fails).
Precision: each tensor fails when its maximum absolute error exceeds ``atol`` (1e-4), its maximum error
relative to the baseline's largest magnitude exceeds ``rtol`` (1e-3) or its cosine similarity falls below
0.999; decoded-image tensors use ``atol`` 2/255 and ``rtol`` 2e-2.  Missing files or tensors and shape
changes fail.  Performance: lower-is-better times (``perf/time_per_step``, ``timing_s/gen``,
``timing_s/old_log_prob``, ``timing_s/reward``, ``timing_s/update_actor``, ``timing_s/update_weights``) fail
when more than the threshold (15 %; 20 % for ``update_weights``) above the baseline, higher-is-better
rates (``perf/throughput``, ``perf/mfu/actor``, ``perf/mfu/actor_infer``) when more than the threshold below.

Counterpart of the reference's nightly single-sample regression (``tests/nightly/qwen_image_flowgrpo``:
README thresholds, test-side debug hooks); here it is a user tool that needs no CI service, and the hooks
wrap the trainer's methods from outside (no production code changes its behaviour).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import sys
from typing import Optional

import torch

LOWER_BETTER = ("perf/time_per_step", "timing_s/gen", "timing_s/old_log_prob", "timing_s/reward",
                "timing_s/update_actor", "timing_s/update_weights")
HIGHER_BETTER = ("perf/throughput", "perf/mfu/actor", "perf/mfu/actor_infer")
WIDE = {"timing_s/update_weights": 0.20}
IMAGE_KEYS = ("batch.responses", "batch.images", "batch.pixels")

DEFAULT_OVERRIDES = [
    "actor_rollout_ref.model.architecture=tiny_dit", "data.train_batch_size=2", "actor_rollout_ref.rollout.n=4",
    "actor_rollout_ref.rollout.pipeline.num_inference_steps=4", "actor_rollout_ref.rollout.algo.noise_level=0.7",
    "actor_rollout_ref.actor.ppo_mini_batch_size=2", "actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu=8",
    "trainer.resume_mode=disable", "trainer.logger=[]", "trainer.save_freq=0",
]


# ------------------------------------------------------------------------------------------ run + dump
def _grad_snapshot(engine) -> dict:
    out = {}
    flats = [f for f in (getattr(engine, "flat", None), getattr(engine, "eflat", None)) if f is not None]
    norms = []
    for f in flats:
        for n, p in zip(f.names, f.params):
            g = getattr(p, "main_grad", None)
            if g is None:
                continue
            if "lora_" in n:
                out[f"gradients.{n}"] = g.detach().float().cpu().clone()
            norms.append(g.detach().float().norm())
    if norms:
        out["grad_norms"] = torch.stack(norms).cpu()
    return out


def run_case(overrides: list[str], out_dir: str, steps: int, dump_steps: set[int]) -> list[dict]:
    """Runs the trainer with dump hooks; writes payloads and ``metrics.jsonl``; returns the step metrics."""
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    cfg = load_config("diffusion_trainer", list(overrides) + [f"trainer.total_training_steps={steps}"])
    D.init_distributed(device=str(cfg.trainer.device))
    t = PolicyGradientTrainer(cfg)
    os.makedirs(out_dir, exist_ok=True)
    state = {"grads": {}}
    train_on, opt_step = t.train_on, t.actor.engine.optimizer_step

    def train_on_hook(out, scores, timer):
        m = train_on(out, scores, timer)
        if t.global_step in dump_steps and D.rank() == 0:
            payload = {f"batch.{k}": v.detach().cpu().clone() for k, v in out.batch.items()
                       if isinstance(v, torch.Tensor) and v.numel() * v.element_size() < (256 << 20)}
            payload["batch.sample_level_scores"] = scores.detach().float().cpu().clone()
            payload.update(state["grads"])
            d = os.path.join(out_dir, f"step_{t.global_step}")
            os.makedirs(d, exist_ok=True)
            torch.save(payload, os.path.join(d, "payload.pt"))
        return m

    def opt_hook(*a, **k):
        if t.global_step in dump_steps:
            state["grads"] = _grad_snapshot(t.actor.engine)  # the last optimizer step of the dumped step wins
        return opt_step(*a, **k)

    t.train_on = train_on_hook
    t.actor.engine.optimizer_step = opt_hook
    hist = []
    with open(os.path.join(out_dir, "metrics.jsonl"), "w") as f:
        for _ in range(steps):
            m = t.step()
            row = {k: (float(v) if isinstance(v, (int, float)) or torch.is_tensor(v) else v) for k, v in m.items()
                   if isinstance(v, (int, float)) or (torch.is_tensor(v) and v.numel() == 1)}
            hist.append(row)
            f.write(json.dumps(row) + "\n")
    return hist


def summarise(hist: list[dict], skip: int) -> dict:
    rows = hist[skip:] if len(hist) > skip else hist[-1:]
    out = {}
    for k in LOWER_BETTER + HIGHER_BETTER:
        vals = [r[k] for r in rows if k in r and math.isfinite(r[k])]
        if vals:
            out[k] = sum(vals) / len(vals)
    out["steps_compared"] = len(rows)
    return out


# ------------------------------------------------------------------------------------------ compare
def tensor_errors(cur: torch.Tensor, base: torch.Tensor) -> dict:
    a, b = cur.detach().double().reshape(-1), base.detach().double().reshape(-1)
    if a.numel() == 0:
        return {"max_abs_err": 0.0, "max_rel_err": 0.0, "cos_sim": 1.0}
    diff = (a - b).abs()
    mab = float(diff.max())
    scale = float(b.abs().max())
    rel = mab / scale if scale > 0 else (0.0 if mab == 0 else math.inf)
    na, nb = float(a.norm()), float(b.norm())
    cos = 1.0 if (na == 0 and nb == 0) else (float(a @ b) / (na * nb) if na > 0 and nb > 0 else 0.0)
    return {"max_abs_err": mab, "max_rel_err": rel, "cos_sim": cos}


def compare_dumps(cur_dir: str, base_dir: str, atol: float = 1e-4, rtol: float = 1e-3, min_cos: float = 0.999,
                  img_atol: float = 2 / 255, img_rtol: float = 2e-2, img_min_cos: float = 0.999) -> dict:
    report = {"ok": True, "files": {}, "failures": []}
    base_files = sorted(d for d in os.listdir(base_dir) if d.startswith("step_")) if os.path.isdir(base_dir) else []
    if not base_files:
        report["ok"] = False
        report["failures"].append("baseline has no step dumps")
    for d in base_files:
        bp, cp = os.path.join(base_dir, d, "payload.pt"), os.path.join(cur_dir, d, "payload.pt")
        if not os.path.exists(cp):
            report["ok"] = False
            report["failures"].append(f"{d}: missing current payload")
            continue
        base, cur = torch.load(bp, weights_only=True), torch.load(cp, weights_only=True)
        res = {}
        for k, bt in base.items():
            if k not in cur:
                report["failures"].append(f"{d}/{k}: missing tensor")
                report["ok"] = False
                continue
            ct = cur[k]
            if tuple(ct.shape) != tuple(bt.shape):
                report["failures"].append(f"{d}/{k}: shape {tuple(ct.shape)} != {tuple(bt.shape)}")
                report["ok"] = False
                continue
            e = tensor_errors(ct, bt)
            img = k in IMAGE_KEYS
            lim = (img_atol, img_rtol, img_min_cos) if img else (atol, rtol, min_cos)
            e["ok"] = bool(e["max_abs_err"] <= lim[0] and e["max_rel_err"] <= lim[1] and e["cos_sim"] >= lim[2])
            if not e["ok"]:
                report["ok"] = False
                report["failures"].append(f"{d}/{k}: abs {e['max_abs_err']:.3g} rel {e['max_rel_err']:.3g} "
                                          f"cos {e['cos_sim']:.6f}")
            res[k] = e
        report["files"][d] = res
    return report


def compare_metrics(cur: dict, base: dict, threshold: float = 0.15) -> dict:
    report = {"ok": True, "metrics": {}, "failures": []}
    for k in LOWER_BETTER + HIGHER_BETTER:
        if k not in base or k not in cur or base[k] == 0:
            continue
        th = WIDE.get(k, threshold)
        change = (cur[k] - base[k]) / abs(base[k])
        bad = change > th if k in LOWER_BETTER else change < -th
        report["metrics"][k] = {"baseline": base[k], "current": cur[k], "rel_change": change, "threshold": th,
                                "ok": not bad}
        if bad:
            report["ok"] = False
            report["failures"].append(f"{k}: {base[k]:.4g} -> {cur[k]:.4g} ({100 * change:+.1f} %)")
    return report


def main(argv: Optional[list[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--case", default="flowgrpo_tiny")
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--dump-steps", default="1,2")
    ap.add_argument("--perf-skip-steps", type=int, default=2)
    ap.add_argument("--perf-threshold", type=float, default=0.15)
    ap.add_argument("--no-perf", action="store_true", help="compare precision only (e.g. on a shared machine)")
    ap.add_argument("--strict", action="store_true", help="fail when no baseline exists instead of creating it")
    a, overrides = ap.parse_known_args(argv)
    device = "cuda" if torch.cuda.is_available() else "cpu"
    ovr = DEFAULT_OVERRIDES + [f"trainer.device={device}"] + overrides
    cur = os.path.join(a.out, "current", a.case)
    base = os.path.join(a.out, "baseline", a.case)
    if a.strict and not os.path.isdir(base):
        print(json.dumps({"ok": False, "error": f"no baseline at {base}"}))
        return 2
    if os.path.isdir(cur):
        shutil.rmtree(cur)
    hist = run_case(ovr, cur, a.steps, {int(s) for s in a.dump_steps.split(",") if s})
    summary = summarise(hist, a.perf_skip_steps)
    with open(os.path.join(cur, "metrics.json"), "w") as f:
        json.dump(summary, f, indent=2)
    if not os.path.isdir(base):
        shutil.copytree(cur, base)
        print(json.dumps({"ok": True, "baseline_created": base}))
        return 0
    dumps = compare_dumps(cur, base)
    with open(os.path.join(cur, "dump_compare.json"), "w") as f:
        json.dump(dumps, f, indent=2)
    ok = dumps["ok"]
    result = {"precision_ok": dumps["ok"], "precision_failures": dumps["failures"][:20]}
    if not a.no_perf:
        with open(os.path.join(base, "metrics.json")) as f:
            perf = compare_metrics(summary, json.load(f), a.perf_threshold)
        with open(os.path.join(cur, "metrics_compare.json"), "w") as f:
            json.dump(perf, f, indent=2)
        ok = ok and perf["ok"]
        result.update({"perf_ok": perf["ok"], "perf_failures": perf["failures"]})
    result["ok"] = ok
    print(json.dumps(result))
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
