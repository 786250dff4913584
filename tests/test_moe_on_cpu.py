"""MoE dispatch plan (sort by expert, 128-row padding, tile table) on CPU."""

import torch

from verl_omni_b200.ops.moe import TILE, moe_ffn_reference, plan_dispatch


def test_plan_dispatch_layout():
    torch.manual_seed(0)
    T, K, E = 300, 4, 16
    idx = torch.stack([torch.randperm(E)[:K] for _ in range(T)])
    p = plan_dispatch(idx, E)
    counts = torch.bincount(idx.reshape(-1), minlength=E)
    seg = p.seg.long()
    assert torch.equal(seg[1:] - seg[:-1], (counts + TILE - 1) // TILE * TILE)
    assert p.rows % TILE == 0 and p.rows >= int(seg[-1])
    # every pair lands inside its expert's segment, rows unique
    e_sorted = idx.reshape(-1)[p.order]
    assert torch.all(p.dst >= seg[e_sorted]) and torch.all(p.dst < seg[e_sorted] + counts[e_sorted])
    assert p.dst.unique().numel() == p.dst.numel()
    assert torch.equal(p.tok, torch.arange(T).repeat_interleave(K)[p.order])
    # tile table: expert of each used tile, -1 after the last expert
    for t in range(p.rows // TILE):
        r = t * TILE
        want = int(torch.searchsorted(seg[1:], torch.tensor(r), right=True)) if r < int(seg[-1]) else -1
        assert int(p.tile_expert[t]) == want


def test_sorted_layout_reproduces_reference():
    """Running each tile's expert on the padded sorted buffer and combining equals the per-expert loop."""
    torch.manual_seed(1)
    T, K, E, D, Fh = 64, 2, 8, 16, 12
    h = torch.randn(T, D)
    idx = torch.stack([torch.randperm(E)[:K] for _ in range(T)])
    gates = torch.softmax(torch.randn(T, K), -1)
    wgu, wd = torch.randn(E, 2 * Fh, D) * 0.1, torch.randn(E, D, Fh) * 0.1
    p = plan_dispatch(idx, E)
    xs = torch.zeros(p.rows, D).index_copy(0, p.dst, h[p.tok])
    y = torch.zeros(p.rows, D)
    for t, e in enumerate(p.tile_expert.tolist()):
        if e < 0:
            continue
        rows = slice(t * TILE, (t + 1) * TILE)
        g, u = (xs[rows] @ wgu[e].t()).chunk(2, -1)
        y[rows] = (torch.nn.functional.silu(g) * u) @ wd[e].t()
    out = torch.zeros(T, D).index_add(0, p.tok, y[p.dst] * gates.reshape(-1)[p.order, None])
    torch.testing.assert_close(out, moe_ffn_reference(h, idx, gates, wgu, wd), rtol=1e-5, atol=1e-5)
