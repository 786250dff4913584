"""FlowGRPO step benchmark: SD3.5-Medium-shaped MMDiT, rollout + reward + train, samples/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (per GPU, weak scaling -- the 8-GPU run is exactly 48 prompts x group 16):
6 prompts x group 16 = 96 samples; 16x64x64 latents (1024 image tokens) + 333 text tokens
(256 T5-style + 77 CLIP-style random embeddings, dim 4096) + pooled 2048-d embedding; 10 SDE
steps (sde, noise 0.7) all trained; random-init frozen VAE decoder -> 512^2 images -> random-init
ViT-B/16 scorer; GRPO advantages; old-log-prob recompute; full fine-tune AdamW (lr 1e-5,
clip 1.0), one optimizer step per FlowGRPO step.  Random-init weights, synthetic data.

Timing: W untimed warm-up steps; K steps bracketed by barrier + cuda.synchronize, CUDA events
on the launching stream, max over ranks.  The end-to-end number runs max(1, K // 2) further steps
through the public trainer API (wall clock, max over ranks) with the prompt inputs copied each step
from pinned host memory and the step's metrics read back to the host; its step count is in its
"steps" key.  "mfu" is the model-FLOPs utilisation of the last timed step by phase (architecture
FLOPs formula over the measured bf16 GEMM peak).  Inputs (weights, activations, trajectories) are far larger
than the 126 MB L2, so no explicit flush is used.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

METRIC = "FlowGRPO step time & samples/sec (rollout+train) at 1/2/4/8 B200, max over ranks"
PROMPTS_PER_GPU = 6
GROUP = 16

# Workloads of the headline metric (global batch at 8 GPUs / 8 = the per-GPU share under weak scaling; with
# sequence parallelism a group of `sp` GPUs shares its samples, so prompts are counted per data-parallel group).
CONFIGS = {
    "sd35": dict(arch="sd35_medium", prompts_per_dp=6, group=16, sde_steps=10, sp=1, micro=16, max_num_seqs=48,
                 model="SD3.5-Medium-shaped MMDiT (2.24B params, 24 joint blocks, hidden 1536, 24 heads, patch 2, "
                       "16-ch latents)", seq_len=1024 + 333,
                 reward="random-init VAE decoder 512^2 + ViT-B/16 scorer"),
    "flux_sp2": dict(arch="flux1_dev", prompts_per_dp=6, group=12, sde_steps=16, sp=2, micro=4, max_num_seqs=12,
                     grad_ckpt=True,
                     model="FLUX.1-dev-shaped rectified-flow transformer (~12B, 19 double + 38 single blocks, hidden "
                           "3072, 24 heads, 2D RoPE), full fine-tune, guidance embedding 3.5", seq_len=4096 + 512,
                     reward="random-init VAE decoder 1024^2 + ViT-B/16 scorer"),
    "wan_sp8_async": dict(arch="wan21_14b", prompts_per_dp=8, group=8, sde_steps=20, sp=8, micro=1, max_num_seqs=4,
                          grad_ckpt=True,
                          model="Wan2.1-14B-shaped video DiT (40 blocks, hidden 5120, 40 heads, FFN 13824, 3D RoPE), "
                                "81 frames 480x832", seq_len=32760 + 512, v1="separate_async",
                          reward="random-init VAE decoder + 12-layer ViT per frame, mean-pooled"),
}


def _clock_sampler(path: str):
    try:
        return subprocess.Popen(
            ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except Exception:  # noqa: BLE001
        return None


def _clock_summary(path: str) -> dict:
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    try:
        for line in open(path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
    except OSError:
        pass
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons)}


_REF_INSTALL = ("python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --target "
                "baseline/_ref <reference source>")


def reference_arm(args) -> None:
    """The reference's own trainer through its public entry point, or one line saying why it cannot run.

    The offline install with dependencies stops at resolution (``accelerate>=1.14.0`` is not in the
    wheelhouse); with ``--no-deps`` it installs, and the import of its trainer names the first missing
    runtime dependency, which is reported here as found on this machine."""
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "verl_omni")):
        why = (f"not installed under baseline/_ref: `{_REF_INSTALL}` fails offline (accelerate>=1.14.0 not in "
               "the wheelhouse); the --no-deps install imports without diffusers/verl/ray/vllm_omni")
    else:
        sys.path.insert(0, ref)
        try:
            import verl_omni.trainer.main_diffusion  # noqa: F401

            why = ("reference imports, but its trainer needs a Ray cluster and vLLM-Omni rollout servers, "
                   "neither installable offline")
        except Exception as e:  # noqa: BLE001
            why = (f"`{_REF_INSTALL} --no-deps` installed it; importing verl_omni.trainer.main_diffusion fails: "
                   f"{type(e).__name__}: {e}".replace("\n", " "))
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def _max_mem_gb(dev, n: int) -> float:
    """Peak bytes held by the caching allocator on any rank (GB), symmetric buffers excluded."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([torch.cuda.max_memory_allocated(dev) / 1e9], dtype=torch.float64, device=dev)
    if n > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return round(float(t.item()), 2)


class _PinnedOnce:
    """Serves one pre-pinned host batch through the dataset interface (end-to-end input path)."""

    def __init__(self, ds, host):
        self.ds, self.host = ds, host

    def get_batch(self, ids):
        return self.host

    def __getattr__(self, k):
        return getattr(self.ds, k)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="sd35", choices=list(CONFIGS) + ["omni_moe"],
                    help="sd35 (default): SD3.5-Medium FSDP-style DP; flux_sp2: FLUX-12B full FT with Ulysses SP=2; "
                         "wan_sp8_async: Wan-14B video with SP=8 and the async trainer; omni_moe: Qwen3-Omni-30B-A3B "
                         "MoE GRPO with EP and TP=2")
    ap.add_argument("--arch", default=None)
    ap.add_argument("--prompts-per-gpu", type=int, default=None, help="prompts per data-parallel group")
    ap.add_argument("--group", type=int, default=None)
    ap.add_argument("--sde-steps", type=int, default=None)
    ap.add_argument("--micro", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None, help="omni_moe: decoder layers (default: the full 48)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-step", action="store_true",
                    help="after warm-up, run one step under torch.profiler and print the top CUDA kernels (no bench line)")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.config == "omni_moe":
        return bench_omni(args)
    C = dict(CONFIGS[args.config])
    for k, a in (("arch", "arch"), ("prompts_per_dp", "prompts_per_gpu"), ("group", "group"),
                 ("sde_steps", "sde_steps"), ("micro", "micro")):
        if getattr(args, a) is not None:
            C[k] = getattr(args, a)

    import torch
    import torch.distributed as dist

    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    info = D.init_distributed(device="cuda", timeout_s=1800)
    N = D.world_size()
    assert N == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={N}"
    sp = min(int(C["sp"]), N)
    dp = N // sp
    prompts = int(C["prompts_per_dp"]) * dp
    ov = [
        "trainer.device=cuda", f"actor_rollout_ref.model.architecture={C['arch']}",
        f"data.train_batch_size={prompts}", f"actor_rollout_ref.rollout.n={C['group']}",
        f"actor_rollout_ref.rollout.pipeline.num_inference_steps={C['sde_steps']}",
        "actor_rollout_ref.rollout.algo.noise_level=0.7", "actor_rollout_ref.rollout.algo.sde_type=sde",
        f"actor_rollout_ref.rollout.max_num_seqs={C['max_num_seqs']}",
        f"actor_rollout_ref.actor.fsdp_config.ulysses_sequence_parallel_size={sp}",
        f"actor_rollout_ref.actor.ppo_mini_batch_size={prompts}",
        f"actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu={C['micro']}",
        "actor_rollout_ref.actor.optim.lr=1e-5", "actor_rollout_ref.actor.optim.weight_decay=0.0",
        "trainer.total_training_steps=1000", "trainer.resume_mode=disable", "trainer.logger=[]",
        "trainer.save_freq=-1",
    ]
    if C.get("grad_ckpt"):  # multi-billion-parameter models at 4-32k tokens: recompute block activations
        ov.append("actor_rollout_ref.model.enable_gradient_checkpointing=true")
    if C.get("v1"):
        ov += ["trainer.use_v1=true", f"trainer.v1.trainer_mode={C['v1']}"]
    cfg = load_config("diffusion_trainer", ov)
    if C.get("v1"):
        from verl_omni_b200.trainer.diffusion.v1.trainer import build_v1_trainer

        v1 = build_v1_trainer(cfg)
        trainer = v1.core
        v1.on_train_begin()
        trainer.step = lambda ids=None: v1.step()  # the async trainer's step through the same driver loop
    else:
        trainer = PolicyGradientTrainer(cfg)
    dev = info.device
    n_params = sum(p.numel() for p in trainer.actor.module.parameters())

    def barrier_sync():
        D.barrier()
        torch.cuda.synchronize()

    t_warm = time.perf_counter()
    for _ in range(args.warmup):
        m = trainer.step()
    t_warm = time.perf_counter() - t_warm
    if info.rank == 0:
        print(json.dumps({"warmup_s": round(t_warm, 2), "timing": {k: round(v, 3) for k, v in m.items()
                                                                   if k.startswith("timing_s/")}}),
              file=sys.stderr, flush=True)
    if args.profile_step:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
            trainer.step()
            torch.cuda.synchronize()
        if info.rank == 0:
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=70))
            # torch-level ops (copies, elementwise) by input shape: where the non-kernel device time goes
            ka = [e for e in prof.key_averages(group_by_input_shape=True) if e.key.startswith("aten::")]
            ka.sort(key=lambda e: -e.device_time_total)
            print("aten ops by input shape (device time, calls):")
            for e in ka[:25]:
                print(f"  {e.device_time_total / 1e3:10.1f} ms  {e.count:7d}  {e.key:28s} {str(e.input_shapes)[:110]}")
        D.destroy()
        return
    # ----------------------------------------------------------- device-timed region
    clock_path = os.path.join(os.environ.get("VO_BENCH_DIR", "/tmp"), f"clocks_{info.rank}.csv")
    sampler = _clock_sampler(clock_path) if info.local_rank == 0 else None
    barrier_sync()
    launches0 = ext().launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        m = trainer.step()
    ev1.record()
    barrier_sync()
    launches = ext().launch_count() - launches0
    dev_ms = ev0.elapsed_time(ev1)
    if sampler is not None:
        sampler.terminate()
        sampler.wait()
    t = torch.tensor([dev_ms], dtype=torch.float64, device=dev)
    if N > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms = float(t.item())
    ms_per_step = dev_ms / args.steps
    samples_per_step = prompts * int(C["group"])
    value = samples_per_step / (ms_per_step / 1000.0)
    timing = {k: round(v, 3) for k, v in m.items() if k.startswith("timing_s/")}
    mfu = {k.split("perf/mfu/")[1]: round(v, 4) for k, v in m.items() if k.startswith("perf/mfu/")}
    # ----------------------------------------------------------- end-to-end through the public API
    e2e = None
    if not args.no_e2e:
        ds = trainer.dataset
        h2d = d2h = 0
        e2e_steps = max(1, args.steps // 2)
        barrier_sync()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ids = trainer.sampler.next_batch()
            host = ds.get_batch(trainer.local_prompt_ids(ids))
            for k in list(host.batch):
                host.batch[k] = host.batch[k].pin_memory()
                h2d += host.batch[k].numel() * host.batch[k].element_size()
            trainer.dataset = _PinnedOnce(ds, host)
            m = trainer.step(ids)
            trainer.dataset = ds
            d2h += 4 * len([v for v in m.values() if isinstance(v, float)])
        barrier_sync()
        wall = time.perf_counter() - t0
        w = torch.tensor([wall], dtype=torch.float64, device=dev)
        if N > 1:
            dist.all_reduce(w, op=dist.ReduceOp.MAX)
        wall = float(w.item())
        e2e = {"value": round(samples_per_step * e2e_steps / wall, 4), "unit": "samples/s",
               "h2d_bytes_per_step": h2d // e2e_steps, "d2h_bytes_per_step": d2h // e2e_steps,
               "ms_per_step": round(1000.0 * wall / e2e_steps, 2), "steps": e2e_steps}
    clocks = _clock_summary(clock_path) if info.local_rank == 0 else None
    mem_gb = _max_mem_gb(dev, N)
    if info.rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 4), "unit": "samples/s", "n_gpus": N, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random prompt embeddings / latents, random-init weights)",
            "config": {"model": C["model"] + f" [{n_params / 1e9:.2f}B params]", "name": args.config,
                       "global_batch": samples_per_step, "prompts": prompts, "group": int(C["group"]),
                       "seq_len": C["seq_len"], "sde_steps": int(C["sde_steps"]),
                       "parallelism": f"dp{dp}" + (f"_sp{sp}" if sp > 1 else ""), "reward": C["reward"],
                       "trainer": C.get("v1", "sync"), "l2": "inputs larger than L2 (no flush)"},
            "impl": "native", "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "phase_s": timing, "mfu": mfu,
            "max_memory_allocated_gb": mem_gb,
        }
        print(json.dumps(out), flush=True)
    D.destroy()


def bench_omni(args) -> None:
    """Qwen3-Omni-30B-A3B-shaped MoE thinker GRPO (48 layers, hidden 2048, 128 experts top-8, vocab 151936):
    512-token multimodal prompts (256 audio frames through the audio tower + 256 image patches through the
    vision tower), 1024-token responses, group 8; EP over all GPUs (experts sharded), TP=2 attention when
    N >= 2; per-GPU share of 64 prompts at 8 GPUs.  Same timing rules and JSON line as the diffusion configs."""
    import torch
    import torch.distributed as dist

    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.trainer.main_omni import build_omni_trainer
    from verl_omni_b200.utils.config import load_config

    info = D.init_distributed(device="cuda", timeout_s=1800)
    N = D.world_size()
    assert N == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={N}"
    tp = 2 if N >= 2 else 1
    dp = N // tp
    per_dp = args.prompts_per_gpu or 16
    group = args.group or 8
    ov = []
    if args.layers:  # full width, fewer decoder layers (a smoke run on few GPUs; named in the config below)
        ov.append(f"actor_rollout_ref.model.num_layers={args.layers}")
    cfg = load_config("omni_trainer", ov + [
        "trainer.device=cuda", f"data.train_batch_size={per_dp * dp}", f"actor_rollout_ref.rollout.n={group}",
        "actor_rollout_ref.rollout.response_length=1024", f"actor_rollout_ref.actor.megatron.expert_model_parallel_size={N}",
        f"actor_rollout_ref.actor.megatron.tensor_model_parallel_size={tp}",
        f"actor_rollout_ref.actor.ppo_micro_batch_size_per_gpu={args.micro or 8}", "trainer.logger=[]",
        "trainer.total_training_steps=1000", "trainer.resume_mode=disable"])
    tr = build_omni_trainer(cfg)

    def sync():
        D.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        m = tr.step(tr.prompts_per_rank)
    sync()
    launches0 = ext().launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        m = tr.step(tr.prompts_per_rank)
    e1.record()
    sync()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=info.device)
    if N > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    samples = per_dp * dp * group
    mem_gb = _max_mem_gb(info.device, N)
    if info.rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(samples / (ms / 1000.0), 4), "unit": "samples/s", "n_gpus": N,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random text ids, log-mel frames, image patches; random-init weights)",
            "config": {"model": "Qwen3-Omni-30B-A3B-shaped MoE thinker (48 layers, hidden 2048, 32 q / 4 kv heads, "
                                "128 experts top-8, expert FFN 768, vocab 151936) + 32-layer audio / 27-layer vision towers",
                       "name": "omni_moe", "global_batch": samples, "prompts": per_dp * dp, "group": group,
                       "layers": args.layers or 48,
                       "seq_len": 512 + 1024, "parallelism": f"ep{N}_tp{tp}_dp{dp}", "reward": "seeded hash of the "
                       "response tokens", "l2": "inputs larger than L2 (no flush)"},
            "impl": "native", "gpu_launches": ext().launch_count() - launches0, "max_memory_allocated_gb": mem_gb,
            "phase_s": {k: round(v, 3) for k, v in m.items() if k.startswith("timing_s/")}}), flush=True)
    D.destroy()


if __name__ == "__main__":
    main()
