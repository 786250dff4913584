"""Tensor + sequence parallel linears (Megatron layout) on gloo ranks: a column-parallel -> row-parallel MLP
over TP=2 equals the single-rank MLP in outputs and gradients."""

import torch

from tests._dist_util import run_ranks


def _mlp_check(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.parallel.tensor_parallel import TPContext, column_parallel_linear, row_parallel_linear

    torch.manual_seed(0)
    S, D, Hd = 8, 16, 24
    x = torch.randn(S, D)
    w1, b1 = torch.randn(Hd, D) * 0.2, torch.randn(Hd) * 0.1
    w2, b2 = torch.randn(D, Hd) * 0.2, torch.randn(D) * 0.1
    gy = torch.randn(S, D)
    # single-rank reference
    leaves = [t.clone().requires_grad_() for t in (x, w1, b1, w2, b2)]
    ref = torch.nn.functional.linear(torch.nn.functional.gelu(torch.nn.functional.linear(leaves[0], leaves[1],
                                                                                         leaves[2])), leaves[3], leaves[4])
    (ref * gy).sum().backward()
    # TP = world: rows of the sequence, output columns of w1, input columns of w2
    tp = TPContext(dist.group.WORLD)
    sl, hl = S // world, Hd // world
    xs = x[rank * sl:(rank + 1) * sl].clone().requires_grad_()
    w1s = w1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
    b1s = b1[rank * hl:(rank + 1) * hl].clone().requires_grad_()
    w2s = w2[:, rank * hl:(rank + 1) * hl].clone().requires_grad_()
    b2r = b2.clone().requires_grad_()
    h = torch.nn.functional.gelu(column_parallel_linear(xs, w1s, b1s, tp))  # [S, Hd/world]
    y = row_parallel_linear(h, w2s, b2r, tp)  # [S/world, D]
    torch.testing.assert_close(y, ref[rank * sl:(rank + 1) * sl].detach(), rtol=1e-5, atol=1e-5)
    (y * gy[rank * sl:(rank + 1) * sl]).sum().backward()
    torch.testing.assert_close(xs.grad, leaves[0].grad[rank * sl:(rank + 1) * sl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(w1s.grad, leaves[1].grad[rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b1s.grad, leaves[2].grad[rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(w2s.grad, leaves[3].grad[:, rank * hl:(rank + 1) * hl], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b2r.grad, leaves[4].grad, rtol=1e-4, atol=1e-5)


def test_tp_mlp_world2_gloo():
    run_ranks(_mlp_check, 2)


def _moe_llm_check(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM
    from verl_omni_b200.parallel.tensor_parallel import TPContext

    torch.manual_seed(0)
    m = MoELLM(MoEConfig.tiny())
    ids = torch.randint(0, 500, (2, 11), generator=torch.Generator().manual_seed(3))  # odd length: padded
    gy = torch.randn(2, 11, m.cfg.vocab, generator=torch.Generator().manual_seed(4))
    ref = m(ids)
    (ref * gy).sum().backward()
    ref_g = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
    m.zero_grad(set_to_none=True)
    m.tp = TPContext(dist.group.WORLD)
    out = m(ids)
    torch.testing.assert_close(out, ref.detach(), rtol=1e-4, atol=1e-5)
    (out * gy).sum().backward()
    for n, p in m.named_parameters():
        if p.grad is None:
            assert n not in ref_g, n
            continue
        g = p.grad.clone()
        dist.all_reduce(g)  # each rank holds its heads' / tokens' share
        torch.testing.assert_close(g, ref_g[n], rtol=1e-3, atol=1e-5, msg=lambda s: f"{n}: {s}")


def test_moe_llm_tensor_parallel_world2_gloo():
    run_ranks(_moe_llm_check, 2)


def _omni_step(rank, world, outdir, tp):
    import torch.distributed as dist

    from verl_omni_b200.models.moe_llm import MoEConfig
    from verl_omni_b200.trainer.omni.omni_trainer import OmniGRPOTrainer
    from verl_omni_b200.workers.config.diffusion import DiffusionActorConfig

    ac = DiffusionActorConfig()
    ac.optim.lr = 1e-3
    t = OmniGRPOTrainer(MoEConfig.tiny(), ac, device=torch.device("cpu"), n=4,
                        tp_group=dist.group.WORLD if tp > 1 else None)
    m = t.step(num_prompts=2)
    if rank == 0:
        torch.save({"w": t.engine.flat.flat.clone(), "loss": m["actor/pg_loss"]}, f"{outdir}/tp{tp}.pt")


def test_omni_grpo_step_tp2_matches_tp1(tmp_path):
    run_ranks(_omni_step, 1, (str(tmp_path), 1))
    run_ranks(_omni_step, 2, (str(tmp_path), 2))
    a, b = torch.load(tmp_path / "tp1.pt"), torch.load(tmp_path / "tp2.pt")
    assert abs(a["loss"] - b["loss"]) < 1e-4
    torch.testing.assert_close(b["w"], a["w"], rtol=1e-3, atol=5e-5)  # Adam normalises near-zero gradients
