"""Fused optimizer collective over symmetric (peer-mapped) memory.

CPU: the host restatement of the two kernels on emulated ranks equals reduce-scatter + clipped
AdamW + all-gather.  2+ GPUs: the IPC-mapped kernels equal the NCCL path of the engine.
"""

import math

import pytest
import torch

from tests._dist_util import run_ranks
from verl_omni_b200.parallel.symm_mem import fused_optimizer_step_reference
from verl_omni_b200.workers.engine.base import _adamw_torch


def _standard(grads, master_full, m_full, v_full, lr, betas, eps, wd, step, max_norm):
    W = len(grads)
    g = sum(x.float() for x in grads) / W
    norm = float(g.double().norm())
    coef = min(1.0, max_norm / (norm + 1e-6))
    p, m, v = master_full.clone(), m_full.clone(), v_full.clone()
    _adamw_torch(p, g * coef, m, v, lr, betas[0], betas[1], eps, wd, step)
    return p, m, v, norm


@pytest.mark.parametrize("W", [2, 4])
def test_fused_step_reference_matches_standard_path(W):
    torch.manual_seed(0)
    P = 1024 * W
    n = P // W
    grads = [torch.randn(P) for _ in range(W)]
    master = torch.randn(P)
    m0, v0 = torch.randn(P) * 0.01, torch.rand(P) * 0.01
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, step=3, max_norm=1.0)
    p_ref, m_ref, v_ref, norm = _standard(grads, master, m0, v0, kw["lr"], kw["betas"], kw["eps"],
                                          kw["weight_decay"], kw["step"], kw["max_norm"])
    flats = [torch.zeros(P, dtype=torch.bfloat16) for _ in range(W)]
    sq_parts = [float((sum(g[r * n:(r + 1) * n] for g in grads) / W).double().pow(2).sum()) for r in range(W)]
    total = sum(sq_parts)
    assert math.isclose(math.sqrt(total), norm, rel_tol=1e-6)
    for r in range(W):
        mr, m_r, v_r = master[r * n:(r + 1) * n].clone(), m0[r * n:(r + 1) * n].clone(), v0[r * n:(r + 1) * n].clone()
        sq = fused_optimizer_step_reference(flats, grads, r * n, n, mr, m_r, v_r, sq_total=total, **kw)
        assert math.isclose(sq, sq_parts[r], rel_tol=1e-6)
        torch.testing.assert_close(mr, p_ref[r * n:(r + 1) * n], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(m_r, m_ref[r * n:(r + 1) * n])
        torch.testing.assert_close(v_r, v_ref[r * n:(r + 1) * n])
    for f in flats:  # every emulated rank holds the full bf16 result
        torch.testing.assert_close(f, p_ref.to(torch.bfloat16))


def _gpu_rank(rank, world):
    import torch.distributed as dist

    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.parallel.symm_mem import SymmetricBuffer, fused_optimizer_step

    dev = torch.device("cuda", rank)
    P = 1 << 20
    n = P // world
    lo = rank * n
    gen = torch.Generator(device="cpu").manual_seed(1234)
    master_full = torch.randn(P, generator=gen).to(dev)
    grads = [torch.randn(P, generator=gen).to(dev) for _ in range(world)]
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=0.5)

    flat = SymmetricBuffer(P, torch.bfloat16, dev)
    gbuf = SymmetricBuffer(P, torch.float32, dev)
    flat.tensor.copy_(master_full.to(torch.bfloat16))
    master = master_full[lo:lo + n].clone()
    m, v, gs = torch.zeros_like(master), torch.zeros_like(master), torch.empty_like(master)
    # NCCL path: reduce-scatter -> sq_norm/all-reduce -> adamw_flat -> all-gather
    flat_ref = master_full.to(torch.bfloat16)
    master_ref, m_ref, v_ref = master.clone(), m.clone(), v.clone()
    for step in (1, 2):
        gbuf.tensor.copy_(grads[rank] * step)
        norm = fused_optimizer_step(flat, gbuf, lo, n, master, gs, m, v, step=step, **kw)
        gs_ref = torch.empty_like(master)
        dist.reduce_scatter_tensor(gs_ref, grads[rank] * step)
        gs_ref.mul_(1.0 / world)
        sq = ext().sq_norm(gs_ref)
        dist.all_reduce(sq)
        ext().adamw_flat(master_ref, gs_ref, m_ref, v_ref, flat_ref[lo:lo + n], kw["lr"], kw["betas"][0],
                         kw["betas"][1], kw["eps"], kw["weight_decay"], step, kw["max_norm"], sq, 1.0)
        full = torch.empty_like(flat_ref)
        dist.all_gather_into_tensor(full, flat_ref[lo:lo + n].clone())
        flat_ref = full
        torch.cuda.synchronize()
        torch.testing.assert_close(norm, sq.sqrt(), rtol=1e-5, atol=0)
        torch.testing.assert_close(gs, gs_ref, rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(master, master_ref, rtol=1e-6, atol=1e-7)
        same = (flat.tensor == flat_ref).float().mean().item()
        assert same > 0.999, same  # bf16 rounding of last-ulp fp32 differences (summation order)
        torch.testing.assert_close(flat.tensor.float(), flat_ref.float(), rtol=1e-2, atol=1e-2)
    flat.close()
    gbuf.close()
    D.barrier()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_fused_step_peer_memory_matches_nccl():
    W = min(torch.cuda.device_count(), 8)  # the 2-, 4- and 8-peer kernel variants, as many as the box has
    run_ranks(_gpu_rank, world=W, device="cuda")
