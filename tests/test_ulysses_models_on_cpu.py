"""Ulysses sequence parallelism through whole models on gloo ranks (SP=2): outputs equal the single-rank
model and the sum of the ranks' parameter gradients equals the single-rank gradient."""

import pytest
import torch

from tests._dist_util import run_ranks

CASES = {
    "sd35_tiny": {"St": 12},
    "sd35_tiny_pad": {"St": 13},   # text not divisible by sp: zero-padded and masked
    "flux_tiny": {"St": 12},
    "qwen_image_tiny": {"St": 12, "mask": True},   # right-padded prompt: segment-major keys + key counts
    "qwen_image_tiny_holes": {"St": 12, "mask": "holes"},  # interleaved valid keys: boolean key mask
    "wan_tiny": {"St": 12},
}


def _inputs(name, St, mask):
    from verl_omni_b200.models.registry import get_arch

    spec = get_arch(name.replace("_pad", "").replace("_holes", ""))
    g = torch.Generator().manual_seed(1)
    B = 2
    x = torch.randn(B, *spec.latent_shape, generator=g)
    t = torch.tensor([700.0, 150.0])
    cond = {}
    for k, s in spec.cond_shapes.items():
        if k.endswith("_mask"):
            m = torch.ones(B, St)
            if mask == "holes":
                m[0, 3:6] = 0
            elif mask:
                m[0, St - 5:] = 0
            cond[k] = m
        elif k == "prompt_embeds":
            cond[k] = torch.randn(B, St, s[-1], generator=g)
        else:
            cond[k] = torch.randn(B, *s, generator=g)
    return spec, x, t, cond


def _run(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.pipelines.model_base import DiffusionModelBase

    for name, kw in CASES.items():
        spec, x, t, cond = _inputs(name, kw["St"], kw.get("mask", False))
        ad = DiffusionModelBase.get(spec.adapter, "flow_grpo")
        torch.manual_seed(0)
        m = spec.build()
        gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2))
        ref = ad.forward(m, x, t, cond)
        (ref * gy).sum().backward()
        ref_g = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
        m.zero_grad(set_to_none=True)
        m.sp_group = dist.group.WORLD
        out = ad.forward(m, x, t, cond)
        torch.testing.assert_close(out, ref.detach(), rtol=1e-4, atol=1e-5, msg=lambda s: f"{name}: {s}")
        (out * gy).sum().backward()
        for n, p in m.named_parameters():
            if p.grad is None:
                assert n not in ref_g, (name, n)
                continue
            gsum = p.grad.clone()
            dist.all_reduce(gsum)
            torch.testing.assert_close(gsum, ref_g[n], rtol=1e-3, atol=1e-5, msg=lambda s: f"{name} {n}: {s}")


def test_models_ulysses_sp2_gloo():
    run_ranks(_run, 2)


def _train(rank, world, outdir, sp):
    from tests.test_e2e_tiny_on_cpu import OVR
    from verl_omni_b200.trainer.diffusion.flow_grpo_trainer import PolicyGradientTrainer
    from verl_omni_b200.utils.config import load_config

    ovr = [o for o in OVR if not o.startswith("actor_rollout_ref.model.architecture")]
    cfg = load_config("diffusion_trainer", ovr + [
        "actor_rollout_ref.model.architecture=sd35_tiny", "data.train_batch_size=4",
        f"actor_rollout_ref.actor.fsdp_config.ulysses_sequence_parallel_size={sp}", "actor_rollout_ref.actor.ppo_mini_batch_size=4",
        f"trainer.default_local_dir={outdir}", "trainer.total_training_steps=1", "trainer.resume_mode=disable"])
    t = PolicyGradientTrainer(cfg)
    m = t.step()
    assert m["perf/total_num_samples"] == 16
    if rank == 0:
        torch.save({"w": t.actor.engine.flat.flat.clone(), "m": m}, f"{outdir}/sp{sp}.pt")


def test_trainer_step_sp2_matches_sp1(tmp_path):
    """FlowGRPO step with SP=2 on two ranks (one data-parallel group) equals the one-rank step."""
    run_ranks(_train, 1, (str(tmp_path), 1))
    run_ranks(_train, 2, (str(tmp_path), 2))
    a, b = torch.load(tmp_path / "sp1.pt"), torch.load(tmp_path / "sp2.pt")
    assert abs(a["m"]["actor/pg_loss"] - b["m"]["actor/pg_loss"]) < 1e-4 * max(1.0, abs(a["m"]["actor/pg_loss"]))
    torch.testing.assert_close(b["w"], a["w"], rtol=1e-4, atol=1e-6)
