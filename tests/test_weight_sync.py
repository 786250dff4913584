"""Trainer -> rollout weight resharding plans (CPU restatement) and the peer-push kernel (2+ GPUs)."""

import pytest
import torch

from tests._dist_util import run_ranks
from verl_omni_b200.parallel.weight_sync import (ParamSpec, execute_plan_reference, plan_replicate, plan_tp,
                                                 rollout_layout)


def _specs():
    shapes = [((64, 32), 0), ((48, 64), 1), ((40,), None), ((16, 8, 8), 0)]
    specs, off = [], 0
    for i, (shape, dim) in enumerate(shapes):
        specs.append(ParamSpec(f"p{i}", shape, off, dim))
        off += (torch.Size(shape).numel() + 15) // 16 * 16  # trainer flat offsets stay 32-byte aligned
    return specs, off


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tp_plan_reassembles_every_shard(tp):
    torch.manual_seed(0)
    specs, numel = _specs()
    src = torch.randn(numel).bfloat16()
    layout, nbytes = rollout_layout(specs, tp)
    dsts = [torch.zeros(nbytes // 2, dtype=torch.bfloat16) for _ in range(tp)]
    execute_plan_reference(src, dsts, plan_tp(specs, tp, list(range(tp))))
    for s in specs:
        full = src[s.offset:s.offset + torch.Size(s.shape).numel()].view(s.shape)
        for d in range(tp):
            o = layout[s.name] // 2
            if s.shard_dim is None:
                got = dsts[d][o:o + full.numel()].view(full.shape)
                torch.testing.assert_close(got, full)
            else:
                part = full.chunk(tp, dim=s.shard_dim)[d]
                got = dsts[d][o:o + part.numel()].view(part.shape)
                torch.testing.assert_close(got, part)


def test_replicate_plan():
    src = torch.randn(1000).bfloat16()
    dsts = [torch.zeros(1000, dtype=torch.bfloat16) for _ in range(3)]
    execute_plan_reference(src, dsts, plan_replicate(2000, [0, 1, 2]))
    for d in dsts:
        assert torch.equal(d, src)


def _gpu_push(rank, world):
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.parallel.symm_mem import SymmetricBuffer
    from verl_omni_b200.parallel.weight_sync import push

    specs, numel = _specs()
    dev = torch.device("cuda", rank)
    tp = world  # every rank is a rollout TP rank; rank 0 also acts as the trainer
    layout, nbytes = rollout_layout(specs, tp)
    buf = SymmetricBuffer(nbytes // 2, torch.bfloat16, dev)
    buf.tensor.zero_()
    torch.manual_seed(0)
    src = torch.randn(numel).bfloat16().to(dev)
    if rank == 0:
        push(src, buf.peer_ptrs, plan_tp(specs, tp, list(range(tp))).to("cpu"))
    else:
        from verl_omni_b200.parallel.symm_mem import stream_barrier

        stream_barrier(None, dev)
    torch.cuda.synchronize()
    ref = [torch.zeros(nbytes // 2, dtype=torch.bfloat16) for _ in range(tp)]
    execute_plan_reference(src.cpu(), ref, plan_tp(specs, tp, list(range(tp))))
    assert torch.equal(buf.tensor.cpu(), ref[rank])
    buf.close()
    D.barrier()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_peer_push_tp_reshard_gpu():
    run_ranks(_gpu_push, world=min(torch.cuda.device_count(), 4), device="cuda")
