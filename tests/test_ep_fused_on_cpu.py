"""Plan of the fused expert-parallel exchange, checked by emulating the peer row copies of W ranks on
the CPU: dispatch lands every routed row in its owner's expert segment, the combine returns every expert
output to the slot of the rank that routed it."""

import numpy as np
import pytest
import torch

from verl_omni_b200.parallel.expert_parallel import _Layout


@pytest.mark.parametrize("W,El", [(2, 2), (4, 3)])
def test_fused_exchange_plan_round_trip(W, El):
    g = torch.Generator().manual_seed(W)
    E, K, D = W * El, 2, 4
    Ts = [int(torch.randint(3, 40, (1,), generator=g)) for _ in range(W)]
    idx = [torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]) for T in Ts]
    h = [torch.randn(T, D, generator=g) for T in Ts]
    C = np.stack([torch.bincount(i.reshape(-1), minlength=E).numpy() for i in idx]).astype(np.int64)
    plans = [_Layout(C, r, El) for r in range(W)]
    cap = int(max(p.rows.max() for p in plans))
    xbuf = [torch.full((cap, D), float("nan")) for _ in range(W)]
    sorted_info = []
    for r in range(W):  # dispatch (the device code's row formulas)
        L = plans[r]
        flat = idx[r].reshape(-1)
        order = torch.argsort(flat, stable=True)
        se = flat[order]
        tok = torch.arange(Ts[r]).repeat_interleave(K)[order]
        dst_rank = se // El
        dst_row = (torch.from_numpy(L.seg_start)[se] + torch.from_numpy(L.src_prefix[r])[se]
                   + (torch.arange(order.numel()) - torch.from_numpy(L.first[r])[se]))
        for i in range(order.numel()):
            xbuf[int(dst_rank[i])][int(dst_row[i])] = h[r][tok[i]]
        sorted_info.append((order, se, tok))
    for r in range(W):  # padding rows are zeroed by the owner
        xbuf[r][torch.from_numpy(plans[r].pad_rows)] = 0.0
    ybuf = [torch.full((int(C[r].sum()), D), float("nan")) for r in range(W)]
    for r in range(W):  # owner: expert e output = x * (e + 1), then combine
        L = plans[r]
        assert L.seg_local[-1] == L.R and L.tile_expert.size == L.R // 128
        assert not torch.isnan(xbuf[r][:L.R]).any()  # every used row written (real or padding)
        for j in range(El):
            lo, hi = int(L.seg_local[j]), int(L.seg_local[j + 1])
            xbuf[r][lo:hi] *= (r * El + j + 1)
        for row, s, slot in zip(L.own_rows, L.own_rank, L.own_slot):
            ybuf[int(s)][int(slot)] = xbuf[r][int(row)]
    for r in range(W):
        order, se, tok = sorted_info[r]
        ref = h[r][tok] * (se[:, None].float() + 1)
        torch.testing.assert_close(ybuf[r], ref)
