"""Job descriptors of the peer-memory Ulysses exchange, replayed on the host for W emulated ranks and
compared with the permute + all-to-all definition of each exchange."""

import pytest
import torch

from verl_omni_b200.parallel import peer_a2a as PA


def _ranks(W, shape, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*shape, generator=g) for _ in range(W)]


@pytest.mark.parametrize("W", [2, 4])
def test_seq_to_head_and_back(W):
    B, H, Sl, Dh = 2, 8, 3, 8
    Hl = H // W
    xs, ys = _ranks(W, (B, H, Sl, Dh), 0), _ranks(W, (B, H, Sl, Dh), 1)
    n = xs[0].numel()
    # two tensors in one exchange: the second lands after the first in the receive slot
    recv = PA.emulate([[PA.s2h_job(xs[r], r, W, 0), PA.s2h_job(ys[r], r, W, n)] for r in range(W)], 2 * n)
    for q in range(W):
        ex = torch.cat([xs[r][:, q * Hl:(q + 1) * Hl] for r in range(W)], 2)
        ey = torch.cat([ys[r][:, q * Hl:(q + 1) * Hl] for r in range(W)], 2)
        assert torch.equal(recv[q][:n].view(B, Hl, W * Sl, Dh), ex)
        assert torch.equal(recv[q][n:].view(B, Hl, W * Sl, Dh), ey)
    # backward: head layout -> sequence layout is the exact inverse
    heads = [recv[q][:n].view(B, Hl, W * Sl, Dh).clone() for q in range(W)]
    back = PA.emulate([[PA.s2h_bwd_job(heads[q], q, W, 0)] for q in range(W)], n)
    for r in range(W):
        assert torch.equal(back[r].view(B, H, Sl, Dh), xs[r])


@pytest.mark.parametrize("W", [2, 4])
def test_head_to_seq_and_back(W):
    B, Sl, F = 2, 5, 8
    os_ = _ranks(W, (B, W * Sl, F), 2)
    n = os_[0].numel()
    recv = PA.emulate([[PA.h2s_job(os_[r], r, W, 0)] for r in range(W)], n)
    for q in range(W):
        ex = torch.cat([os_[r][:, q * Sl:(q + 1) * Sl] for r in range(W)], 2)
        assert torch.equal(recv[q].view(B, Sl, W * F), ex)
    toks = [recv[q].view(B, Sl, W * F).clone() for q in range(W)]
    back = PA.emulate([[PA.h2s_bwd_job(toks[q], q, W, 0)] for q in range(W)], n)
    for r in range(W):
        assert torch.equal(back[r].view(B, W * Sl, F), os_[r])


def test_disabled_without_nccl_group():
    x = torch.zeros(2, 4, 8, 8, dtype=torch.bfloat16)
    assert not PA.applies(None, [x])
