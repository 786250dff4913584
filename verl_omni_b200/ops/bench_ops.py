"""Kernel microbenchmarks: ``python -m verl_omni_b200.ops.bench_ops {gemm,fmha,sde,adaln} [options]``.

Times each op with CUDA events on the launching stream after warm-up (synchronised on both sides),
reports achieved TFLOP/s or GB/s and the fraction of the measured peaks (``MEASURED_PEAKS.json``:
cuBLAS bf16 GEMM burst and STREAM-style copy bandwidth).  ``--compare`` also times the library
equivalent (cuBLAS via ``torch.matmul`` / SDPA) on the same inputs.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch


def _peaks() -> dict:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"tflops": d["bf16_tflops"], "gbs": d["hbm_gbs"], "src": "measured"}
    except OSError:
        return {"tflops": 1590.0, "gbs": 6650.0, "src": "fallback"}


def timeit(fn, iters: int = 10, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def bench_gemm(a) -> list[dict]:
    from verl_omni_b200.ops._ext import ext

    e = ext()
    M, N, K = a.M, a.N, a.K
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    dy = torch.randn(M, N, device="cuda").bfloat16()
    gw = torch.zeros(N, K, device="cuda")
    flops = 2.0 * M * N * K
    cases = {
        "fwd": lambda: e.gemm_fwd(x, w, None, 0, None, None, 1),
        "dgrad": lambda: e.gemm_dgrad(dy, w),
        "wgrad": lambda: e.gemm_wgrad(dy, x, gw, True),
    }
    if a.compare:
        cases["cublas_fwd"] = lambda: torch.matmul(x, w.t())
        cases["cublas_dgrad"] = lambda: torch.matmul(dy, w)
        cases["cublas_wgrad"] = lambda: torch.matmul(dy.t(), x)
    out = []
    for name in a.only.split(",") if a.only else cases:
        ms = timeit(cases[name], a.iters)
        out.append({"op": f"gemm_{name}", "M": M, "N": N, "K": K, "ms": round(ms, 4),
                    "tflops": round(flops / ms / 1e9, 1)})
    return out


# (name, M, N, K) of the linear layers of one SD3.5-Medium-shaped joint block for a 16-sample
# micro-batch (1024 image + 333 text tokens per sample), plus the 48-sample rollout batch
SD35_SHAPES = [
    ("img_qkv", 16 * 1024, 4608, 1536), ("img_out", 16 * 1024, 1536, 1536), ("img_ff1", 16 * 1024, 6144, 1536),
    ("img_ff2", 16 * 1024, 1536, 6144), ("txt_qkv", 16 * 333, 4608, 1536), ("txt_out", 16 * 333, 1536, 1536),
    ("txt_ff1", 16 * 333, 6144, 1536), ("txt_ff2", 16 * 333, 1536, 6144), ("mod", 16, 13824, 1536),
    ("roll_ff1", 48 * 1024, 6144, 1536), ("roll_txt_qkv", 48 * 333, 4608, 1536),
]


def bench_gemm_sweep(a) -> list[dict]:
    """Native tcgen05 GEMM vs cuBLAS on every linear-layer shape of the flagship workload."""
    from verl_omni_b200.ops._ext import ext

    e = ext()
    out = []
    for name, M, N, K in SD35_SHAPES:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
        dy = torch.randn(M, N, device="cuda").bfloat16()
        gw = torch.zeros(N, K, device="cuda")
        row = {"op": "gemm_sweep", "name": name, "M": M, "N": N, "K": K}
        for kind, nat, ref in (
                ("fwd", lambda: e.gemm_fwd(x, w, None, 0, None, None, 1), lambda: torch.matmul(x, w.t())),
                ("dgrad", lambda: e.gemm_dgrad(dy, w), lambda: torch.matmul(dy, w)),
                ("wgrad", lambda: e.gemm_wgrad(dy, x, gw, True), lambda: gw.add_(torch.matmul(dy.t(), x)))):
            tn, tr = timeit(nat, a.iters), timeit(ref, a.iters)
            row[kind] = {"native_ms": round(tn, 4), "cublas_ms": round(tr, 4),
                         "native_tflops": round(2.0 * M * N * K / tn / 1e9, 1)}
        out.append(row)
        del x, w, dy, gw
    return out


# image / text stream pairs of the joint blocks (16 samples x 1024 image + 333 text tokens)
SD35_PAIRS = [("qkv", 4608, 1536), ("out", 1536, 1536), ("ff1", 6144, 1536), ("ff2", 1536, 6144)]


def bench_gemm_pair(a) -> list[dict]:
    """Image + text linears as one grouped launch vs two launches (forward / dgrad / wgrad)."""
    from verl_omni_b200.ops._ext import ext

    e = ext()
    Mi, Mt = 16 * 1024, 16 * 333
    out = []
    for name, N, K in SD35_PAIRS:
        xs = [torch.randn(M, K, device="cuda").bfloat16() for M in (Mi, Mt)]
        ws = [(torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16() for _ in range(2)]
        dys = [torch.randn(M, N, device="cuda").bfloat16() for M in (Mi, Mt)]
        gws = [torch.zeros(N, K, device="cuda") for _ in range(2)]
        flops = 2.0 * (Mi + Mt) * N * K
        row = {"op": "gemm_pair", "name": name, "M": [Mi, Mt], "N": N, "K": K}
        for kind, pair, two in (
                ("fwd", lambda: e.gemm_fwd_pair(xs[0], ws[0], None, None, None, 1, xs[1], ws[1], None, None, None, 1, 0),
                 lambda: (e.gemm_fwd(xs[0], ws[0], None, 0, None, None, 1), e.gemm_fwd(xs[1], ws[1], None, 0, None, None, 1))),
                ("dgrad", lambda: e.gemm_dgrad_pair(dys[0], ws[0], dys[1], ws[1]),
                 lambda: (e.gemm_dgrad(dys[0], ws[0]), e.gemm_dgrad(dys[1], ws[1]))),
                ("wgrad", lambda: e.gemm_wgrad_pair(dys[0], xs[0], gws[0], dys[1], xs[1], gws[1], True),
                 lambda: (e.gemm_wgrad(dys[0], xs[0], gws[0], True), e.gemm_wgrad(dys[1], xs[1], gws[1], True)))):
            tp, tt = timeit(pair, a.iters), timeit(two, a.iters)
            row[kind] = {"pair_ms": round(tp, 4), "two_launch_ms": round(tt, 4), "pair_tflops": round(flops / tp / 1e9, 1),
                         "speedup": round(tt / tp, 3)}
        out.append(row)
    return out


def bench_ulysses(a) -> list[dict]:
    """One joint-attention layer under Ulysses SP (run under torchrun, one rank per GPU): NCCL all-to-all
    path vs the fused path (QKV GEMM epilogue scatter + attention peer output).  FLUX-shaped by default:
    ``--B 1 --S 4096`` image tokens + 512 text tokens, hidden 3072, 24 heads.  Device time of the slowest
    rank; roofline = max(FLOPs / measured GEMM peak, bytes that cross NVLink per GPU / 770 GB/s)."""
    import os

    import torch.distributed as dist

    from verl_omni_b200.models.layers import Linear
    from verl_omni_b200.ops.norm import qk_norm_split_into
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.parallel import ulysses_fused as UF
    from verl_omni_b200.parallel.ulysses import joint_attention

    info = D.init_distributed(device="cuda", timeout_s=300)
    W, dev, grp = D.world_size(), info.device, dist.group.WORLD
    B, Si, St, Dm, H = a.B, a.S, 512, 3072, 24
    dh, si, st = Dm // H, Si // W, St // W
    torch.manual_seed(0)
    qi, qt = Linear(Dm, 3 * Dm).to(dev, torch.bfloat16), Linear(Dm, 3 * Dm).to(dev, torch.bfloat16)
    wn = [torch.ones(dh, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    hi = torch.randn(B, si, Dm, device=dev, dtype=torch.bfloat16)
    ht = torch.randn(B, st, Dm, device=dev, dtype=torch.bfloat16)

    def nccl():
        a0, a1 = qi(hi).reshape(B * si, 3 * Dm), qt(ht).reshape(B * st, 3 * Dm)
        mk = lambda: torch.empty(B, H, si + st, dh, device=dev, dtype=torch.bfloat16)  # noqa: E731
        q, k, v = qk_norm_split_into(mk(), mk(), mk(), a0, wn[0], wn[1], si, 0)
        q, k, v = qk_norm_split_into(q, k, v, a1, wn[2], wn[3], st, si)
        return joint_attention(q, k, v, si, sp_group=grp)

    def fused():
        return UF.joint_attention_fused(hi, ht, qi, qt, (wn[0], wn[1]), (wn[2], wn[3]), H, grp)

    rows = []
    with torch.no_grad():
        for name, fn in (("nccl_all_to_all", nccl), ("fused_peer", fused)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            S = Si + St
            flops = 2.0 * B * (si + st) * Dm * 3 * Dm + 4.0 * B * (H // W) * S * S * dh
            xbytes = 2.0 * B * (si + st) * (3 * Dm + Dm) * (W - 1) / W
            t_roof = max(flops / 1.59e15, xbytes / 770e9) * 1e3
            rows.append({"op": f"ulysses_{name}", "world": W, "B": B, "S_img": Si, "S_txt": St, "hidden": Dm,
                         "ms": round(float(ms), 4), "tflops": round(flops / float(ms) / 1e9, 1),
                         "nvlink_gb": round(xbytes / 1e9, 3), "roofline_ms": round(t_roof, 4),
                         "frac_of_roofline": round(t_roof / float(ms), 3)})
    # training: forward + backward of the same layer; the exchanges as NCCL all-to-alls with permute copies
    # vs one peer-memory kernel each (sequence -> heads for q/k/v, heads -> sequence, and their inverses)
    from verl_omni_b200.parallel import peer_a2a as PA

    hig, htg = hi.clone().requires_grad_(True), ht.clone().requires_grad_(True)
    goi = torch.randn(B, si, Dm, device=dev, dtype=torch.bfloat16)
    got = torch.randn(B, st, Dm, device=dev, dtype=torch.bfloat16)

    def train():
        a0, a1 = qi(hig).reshape(B * si, 3 * Dm), qt(htg).reshape(B * st, 3 * Dm)
        mk = lambda: torch.empty(B, H, si + st, dh, device=dev, dtype=torch.bfloat16)  # noqa: E731
        q, k, v = qk_norm_split_into(mk(), mk(), mk(), a0, wn[0], wn[1], si, 0)
        q, k, v = qk_norm_split_into(q, k, v, a1, wn[2], wn[3], st, si)
        oi, ot = joint_attention(q, k, v, si, sp_group=grp)
        torch.autograd.backward([oi, ot], [goi, got])

    for name, peer in (("train_nccl_all_to_all", "0"), ("train_peer_a2a", "1")):
        os.environ["VO_ULYSSES_PEER"] = peer
        for _ in range(3):
            train()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.iters):
            train()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        S = Si + St
        flops = 3 * 2.0 * B * (si + st) * Dm * 3 * Dm + 3.5 * 4.0 * B * (H // W) * S * S * dh
        xbytes = 2 * 2.0 * B * (si + st) * (3 * Dm + Dm) * (W - 1) / W
        rows.append({"op": f"ulysses_{name}", "world": W, "B": B, "S_img": Si, "S_txt": St, "hidden": Dm,
                     "ms": round(float(ms), 4), "tflops": round(flops / float(ms) / 1e9, 1),
                     "nvlink_gb": round(xbytes / 1e9, 3)})
    os.environ["VO_ULYSSES_PEER"] = "1"
    PA.release_all()
    UF.release_all()
    if D.rank() != 0:
        return []
    return rows


def bench_tp(a) -> list[dict]:
    """Tensor + sequence parallel attention projections of the Qwen3-Omni-30B-A3B thinker shape (hidden 2048,
    32 x 128 query heads) over ``--S`` tokens (run under torchrun): column-parallel q projection (all-gather
    -> GEMM) and row-parallel output projection (GEMM -> reduce-scatter), forward; NCCL collectives around
    tcgen05 GEMMs vs the fused kernels.  Roofline = max(FLOPs / measured GEMM peak, NVLink bytes / 770 GB/s)."""
    import os

    import torch.distributed as dist

    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.parallel.tensor_parallel import TPContext, column_parallel_linear, row_parallel_linear

    D.init_distributed(device="cuda", timeout_s=300)
    W, dev = D.world_size(), torch.device("cuda", torch.cuda.current_device())
    S, Dm, Q = a.S, 2048, 4096
    torch.manual_seed(0)
    x = torch.randn(S // W, Dm, device=dev, dtype=torch.bfloat16)
    wq = (torch.randn(Q // W, Dm, device=dev) * 0.02).bfloat16()
    wo = (torch.randn(Dm, Q // W, device=dev) * 0.02).bfloat16()
    tp = TPContext(dist.group.WORLD)
    rows = []
    with torch.no_grad():
        for name, fused in (("nccl", "0"), ("fused_peer_tma_gather", "kernel"), ("fused_peer", "1")):
            os.environ["VO_TP_FUSED"] = fused

            def step():
                return row_parallel_linear(column_parallel_linear(x, wq, None, tp), wo, None, tp)

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                step()
            e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            flops = 2.0 * 2 * S * Dm * (Q // W)
            xbytes = (W - 1) / W * S * Dm * (2 + 2)  # gathered bf16 activations in, bf16 partial sums out
            t_roof = max(flops / 1.59e15, xbytes / 770e9) * 1e3
            rows.append({"op": f"tp_attn_proj_{name}", "world": W, "tokens": S, "hidden": Dm, "ms": round(float(ms), 4),
                         "tflops": round(flops / float(ms) / 1e9, 1), "roofline_ms": round(t_roof, 4),
                         "frac_of_roofline": round(t_roof / float(ms), 3)})
    tp.release()
    return rows if D.rank() == 0 else []


def bench_optstep(a) -> list[dict]:
    """Sharded optimizer step over ``--numel`` parameters on every rank (run under torchrun):
    NCCL reduce-scatter + AdamW + all-gather vs the fused peer-memory kernels.  Device time of the
    slowest rank; roofline = bytes that must cross NVLink per GPU / measured peer bandwidth."""
    import torch.distributed as dist

    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.parallel import dist as D
    from verl_omni_b200.parallel.symm_mem import SymmetricBuffer, fused_optimizer_step

    info = D.init_distributed(device="cuda", timeout_s=300)
    W, dev = D.world_size(), info.device
    P = (a.numel + 128 * W - 1) // (128 * W) * 128 * W
    n, lo = P // W, (P // W) * D.rank()
    flat = SymmetricBuffer(P, torch.bfloat16, dev)
    grad = SymmetricBuffer(P, torch.float32, dev)
    grad.tensor.normal_()
    master = torch.randn(n, device=dev)
    m, v, gs = torch.zeros_like(master), torch.zeros_like(master), torch.empty_like(master)
    kw = dict(lr=1e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, max_norm=1.0)

    def nccl_step(step):
        dist.reduce_scatter_tensor(gs, grad.tensor)
        gs.mul_(1.0 / W)
        sq = ext().sq_norm(gs)
        dist.all_reduce(sq)
        ext().adamw_flat(master, gs, m, v, flat.tensor[lo:lo + n], kw["lr"], 0.9, 0.999, 1e-8, 0.0, step, 1.0, sq, 1.0)
        dist.all_gather_into_tensor(flat.tensor, flat.tensor[lo:lo + n].clone())

    def fused_step(step):
        fused_optimizer_step(flat, grad, lo, n, master, gs, m, v, step=step, **kw)

    out = []
    for name, fn in (("nccl", nccl_step), ("fused_peer", fused_step)):
        for s in range(3):
            fn(s + 1)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(a.iters):
            fn(s + 4)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        # per GPU over NVLink: fp32 grads of the other shards in, bf16 of own shard to W-1 peers out
        link_bytes = (W - 1) * n * 4 + (W - 1) * n * 2
        out.append({"op": f"optstep_{name}", "world": W, "params": P, "ms": round(float(ms), 3),
                    "link_gbs": round(link_bytes / float(ms) / 1e6, 1),
                    "frac_of_770gbs_link": round(link_bytes / float(ms) / 1e6 / 770.0, 3)})
    flat.close()
    grad.close()
    if D.rank() != 0:
        return []
    return out


def bench_fmha(a) -> list[dict]:
    from verl_omni_b200.ops._ext import ext

    e = ext()
    B, H, S, D = a.B, a.H, a.S, a.D
    q, k, v = (torch.randn(B, H, S, D, device="cuda").bfloat16() for _ in range(3))
    scale = 1 / math.sqrt(D)
    o, lse = e.fmha_fwd(q, k, v, False, scale, 1)
    do = torch.randn_like(o)
    flops_f = 4.0 * B * H * S * S * D
    cases = {"fwd": (lambda: e.fmha_fwd(q, k, v, False, scale, 1), flops_f),
             "fwd2": (lambda: e.fmha_fwd(q, k, v, False, scale, 2), flops_f),
             "fwd3": (lambda: e.fmha_fwd(q, k, v, False, scale, 3), flops_f),
             "fwd4": (lambda: e.fmha_fwd(q, k, v, False, scale, 4), flops_f),
             "fwd5": (lambda: e.fmha_fwd(q, k, v, False, scale, 5), flops_f)}
    for emu in (0, 1, 2, 3, 4):  # version 4 with emu of every 8 exponential pairs on the FMA pipe
        cases[f"fwd4e{emu}"] = (lambda emu=emu: e.fmha_fwd(q, k, v, False, scale, 40 + emu), flops_f)
    if hasattr(e, "fmha_bwd"):
        cases["bwd"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 1), 2.5 * flops_f)
        cases["bwd2"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 2), 2.5 * flops_f)
        cases["bwd3"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 3), 2.5 * flops_f)
        cases["bwd4"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 4), 2.5 * flops_f)
        cases["bwd5"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 5), 2.5 * flops_f)
        cases["bwd7"] = (lambda: e.fmha_bwd(q, k, v, o, lse, do, False, scale, 7), 2.5 * flops_f)
    if a.compare:
        cases["sdpa_fwd"] = (lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v), flops_f)
        qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        og = torch.nn.functional.scaled_dot_product_attention(qg, kg, vg)
        gdo = torch.randn_like(og)
        # backward only: one autograd.grad through the retained SDPA graph per call
        cases["sdpa_bwd"] = (lambda: torch.autograd.grad(og, (qg, kg, vg), gdo, retain_graph=True), 2.5 * flops_f)
    if a.only:
        cases = {k: cases[k] for k in a.only.split(",")}
    out = []
    for name, (fn, fl) in cases.items():
        ms = timeit(fn, a.iters)
        out.append({"op": f"fmha_{name}", "B": B, "H": H, "S": S, "D": D, "ms": round(ms, 4),
                    "tflops": round(fl / ms / 1e9, 1)})
    return out


def bench_sde(a) -> list[dict]:
    from verl_omni_b200.ops.sde import sde_step

    B = a.B
    x = torch.randn(B, 16, 64, 64, device="cuda")
    v = torch.randn_like(x)
    sig = torch.full((B,), 0.6, device="cuda")
    ms = timeit(lambda: sde_step(x, v, sig, sig - 0.1, sigma_max=0.95, noise_level=0.7, seed=1), a.iters)
    nbytes = 4 * x.numel() * 4  # read x, v; write mean, prev
    return [{"op": "sde_step", "B": B, "ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1)}]


def bench_adaln(a) -> list[dict]:
    from verl_omni_b200.ops._ext import ext

    B, S, D = a.B, a.S, 1536
    x = torch.randn(B, S, D, device="cuda").bfloat16()
    mod = torch.randn(B, 6 * D, device="cuda").bfloat16()
    ms = timeit(lambda: ext().adaln_ln_fwd(x, mod, 0, D, None, None, S, 1e-6), a.iters)
    nbytes = 2 * 2 * x.numel()
    return [{"op": "adaln_ln_fwd", "B": B, "S": S, "D": D, "ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1)}]


def bench_moe(a) -> list[dict]:
    """Qwen3-Omni-30B-A3B-shaped MoE layer (128 experts, top-8, hidden 2048, expert FFN 768) on ``--B`` x
    ``--S`` tokens: the expert-grouped GEMMs (one launch per projection) vs a per-expert cuBLAS loop."""
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.ops.moe import plan_dispatch

    E, K, D, Fh = 128, 8, 2048, 768
    T = a.B * a.S
    torch.manual_seed(0)
    idx = torch.topk(torch.randn(T, E, device="cuda"), K, dim=-1).indices
    plan = plan_dispatch(idx, E)
    x = torch.randn(plan.rows, D, device="cuda").bfloat16()
    w = (torch.randn(E, 2 * Fh, D, device="cuda") / D ** 0.5).bfloat16()
    e = ext()
    ms = timeit(lambda: e.moe_gemm_fwd(x, w, plan.tile_expert), a.iters)
    flops = 2.0 * T * K * 2 * Fh * D
    seg = plan.seg.tolist()

    def loop():
        for i in range(E):
            if seg[i + 1] > seg[i]:
                torch.matmul(x[seg[i]:seg[i + 1]], w[i].t())

    ms_loop = timeit(loop, a.iters)
    return [{"op": "moe_grouped_gemm_fwd", "tokens": T, "experts": E, "top_k": K, "N": 2 * Fh, "K": D,
             "padded_rows": int(seg[-1]), "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
             "cublas_per_expert_loop_ms": round(ms_loop, 4)}]


def bench_decode(a) -> list[dict]:
    """Grouped-query decode attention, Qwen3-Omni-30B-A3B thinker heads (32 query / 4 KV heads, head_dim 128):
    ``--B`` sequences with ``--S`` cached positions each, contiguous cache vs paged cache (16-row blocks,
    blocks shuffled across the pool).  Bandwidth counts the K and V bytes read once (the cache is larger
    than L2 at the default sizes)."""
    from verl_omni_b200.ops.decode import decode_attention

    B, L, Hk, rep, hd, bs = a.B, a.S, 4, 8, 128, 16
    q = torch.randn(B, Hk * rep, hd, device="cuda").bfloat16()
    kc = torch.randn(B, Hk, L, hd, device="cuda").bfloat16()
    vc = torch.randn(B, Hk, L, hd, device="cuda").bfloat16()
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    nb = B * L // bs
    perm = torch.randperm(nb, device="cuda")
    # the same rows scattered over a shuffled block pool [blocks, Hk, 16, hd]
    kp = torch.empty(nb, Hk, bs, hd, device="cuda", dtype=torch.bfloat16)
    vp = torch.empty_like(kp)
    kp[perm] = kc.view(B, Hk, L // bs, bs, hd).permute(0, 2, 1, 3, 4).reshape(nb, Hk, bs, hd)
    vp[perm] = vc.view(B, Hk, L // bs, bs, hd).permute(0, 2, 1, 3, 4).reshape(nb, Hk, bs, hd)
    table = perm.view(B, L // bs).to(torch.int32)
    import os

    nbytes = 2 * B * Hk * L * hd * 2
    out = []
    for kernel in ("tcgen05", "cuda_core"):  # VO_DECODE_TC=0 selects the CUDA-core kernel
        os.environ["VO_DECODE_TC"] = "1" if kernel == "tcgen05" else "0"
        kp128 = kc.view(B, Hk, L // 128, 128, hd).permute(0, 2, 1, 3, 4).reshape(B * L // 128, Hk, 128, hd)
        vp128 = vc.view(B, Hk, L // 128, 128, hd).permute(0, 2, 1, 3, 4).reshape(B * L // 128, Hk, 128, hd)
        t128 = torch.arange(B * L // 128, device="cuda", dtype=torch.int32).view(B, L // 128)
        for name, fn in (("contiguous", lambda sp: decode_attention(q, kc, vc, lens, splits=sp)),
                         ("paged16", lambda sp: decode_attention(q, kp, vp, lens, splits=sp, block_table=table)),
                         ("paged128", lambda sp: decode_attention(q, kp128, vp128, lens, splits=sp, block_table=t128))):
            if a.only and name not in a.only.split(","):
                continue
            for sp in ([0] if not a.compare else [0, 1, 2, 4, 8]):  # 0: the default split heuristic
                ms = timeit(lambda: fn(sp), a.iters)
                out.append({"op": f"decode_attn_{name}", "kernel": kernel, "splits": sp or "auto", "B": B, "ctx": L,
                            "q_heads": Hk * rep, "kv_heads": Hk, "hd": hd, "ms": round(ms, 4),
                            "gbs": round(nbytes / ms / 1e6, 1)})
    os.environ["VO_DECODE_TC"] = "1"
    return out


def bench_rollout_decode(a) -> list[dict]:
    """Thinker decode steps at full Qwen3-Omni-30B-A3B width (hidden 2048, 32 / 4 heads of 128, 128 experts,
    top-8, vocab 151936) with ``--layers`` layers: ``--B`` sequences, ``--S``-token prompts, greedy.  The time
    per decode step is (generate with ``--new`` tokens - generate with 1 token) / (``--new`` - 1), eager steps
    vs the step captured as one CUDA graph (``VO_DECODE_GRAPH``)."""
    import os

    from verl_omni_b200.models.moe_llm import MoEConfig, MoELLM
    from verl_omni_b200.utils.dataproto import DataProto
    from verl_omni_b200.workers.rollout.llm_rollout import LLMRolloutEngine

    cfg = MoEConfig(layers=a.layers, audio_layers=1, vision_layers=1)
    torch.manual_seed(0)
    with torch.device("cuda"):
        m = MoELLM(cfg).to(torch.bfloat16).eval()
    batch = DataProto({"input_ids": torch.randint(0, 150000, (a.B, a.S))}, {})
    out = []
    for mode in ("0", "1"):
        os.environ["VO_DECODE_GRAPH"] = mode
        t = {}
        for n in (1, a.new):
            eng = LLMRolloutEngine(m, max_new_tokens=n, temperature=0.0, device=torch.device("cuda"))
            t[n] = timeit(lambda: eng.generate(batch, seed=0), max(2, a.iters // 4), warmup=1)
        step = (t[a.new] - t[1]) / (a.new - 1)
        out.append({"op": "rollout_decode_step", "graph": mode == "1", "layers": a.layers, "B": a.B, "prompt": a.S,
                    "new_tokens": a.new, "ms_per_step": round(step, 3), "ms_per_layer": round(step / a.layers, 4)})
    os.environ["VO_DECODE_GRAPH"] = "1"
    return out


def bench_rowops(a) -> list[dict]:
    """The memory-bound kernels of a training step, each on inputs larger than L2 (126 MB), bytes counted as
    the algorithmic reads + writes: AdaLN LayerNorm forward (D 1536), fused q/k RMSNorm + RoPE + QKV split
    (joint-attention buffers, head_dim 64), flow-matching SDE step with log-prob, RMSNorm (D 2048), SwiGLU,
    per-head RMSNorm + RoPE of the thinker (forward and backward), the linear-backward prologue (GELU' scaling
    + bias-gradient sums over 32768 x 6144), sharded AdamW over a flat fp32 buffer.  ``--iters 1`` for one
    launch of each (ncu captures)."""
    from verl_omni_b200.ops import llm as LO
    from verl_omni_b200.ops._ext import ext
    from verl_omni_b200.ops.norm import qk_norm_split_into
    from verl_omni_b200.ops.sde import sde_step

    out = []
    dev = "cuda"

    def add(op, nbytes, fn, **kw):
        with torch.no_grad():
            ms = timeit(fn, a.iters, warmup=0 if a.iters == 1 else 3)  # --iters 1: one launch (ncu)
        out.append({"op": op, **kw, "ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1)})

    rows, D = 65536, 1536
    x = torch.randn(rows // 16, 16, D, device=dev).bfloat16().view(16, rows // 16, D)
    mod = torch.randn(16, 6 * D, device=dev).bfloat16()
    add("adaln_ln_fwd", 2 * 2 * x.numel(), lambda: ext().adaln_ln_fwd(x, mod, 0, D, None, None, rows // 16, 1e-6),
        rows=rows, D=D)
    B, S, H, Dh = 16, 2048, 24, 64
    x2d = torch.randn(B * S, 3 * H * Dh, device=dev).bfloat16()
    q, k, v = (torch.empty(B, H, S, Dh, device=dev, dtype=torch.bfloat16) for _ in range(3))
    wq, wk = torch.ones(Dh, device=dev).bfloat16(), torch.ones(Dh, device=dev).bfloat16()
    cos, sin = torch.rand(S, Dh // 2, device=dev), torch.rand(S, Dh // 2, device=dev)
    add("qk_rmsnorm_rope_split", 2 * 2 * x2d.numel(),
        lambda: qk_norm_split_into(q, k, v, x2d, wq, wk, S, 0, rope=(cos, sin)), rows=B * S, heads=H, hd=Dh)
    lat = torch.randn(512, 16, 64, 64, device=dev)
    vel = torch.randn_like(lat)
    sig = torch.full((512,), 0.6, device=dev)
    add("sde_step_logprob", 4 * 4 * lat.numel(),
        lambda: sde_step(lat, vel, sig, sig - 0.1, sigma_max=0.95, noise_level=0.7, seed=1), B=512)
    xr = torch.randn(65536, 2048, device=dev).bfloat16()
    w = torch.ones(2048, device=dev).bfloat16()
    add("rms_norm_fwd", 2 * 2 * xr.numel(), lambda: LO.rms_norm(xr, w, 1e-6), rows=65536, D=2048)
    gu = torch.randn(65536, 2 * 768, device=dev).bfloat16()
    add("swiglu_fwd", 2 * gu.numel() + gu.numel(), lambda: LO.swiglu(gu), rows=65536, F=768)
    y = torch.randn(32, 2048, (32 + 4) * 128, device=dev).bfloat16()
    wh = torch.ones(128, device=dev).bfloat16()
    c2, s2 = torch.rand(2048, 64, device=dev), torch.rand(2048, 64, device=dev)
    add("head_rmsnorm_rope", 2 * 2 * 32 * 2048 * 32 * 128, lambda: LO.head_norm_rope(y, 0, 32, wh, c2, s2, 1e-6),
        B=32, S=2048, heads=32, hd=128)
    dyh = torch.randn(32, 32, 2048, 128, device=dev).bfloat16()
    dwh = torch.zeros(128, device=dev)
    add("head_rmsnorm_rope_bwd", 3 * 2 * 32 * 2048 * 32 * 128,
        lambda: ext().head_rmsnorm_rope_bwd(dyh, y, 0, 32, wh, c2, s2, 1e-6, dwh), B=32, S=2048, heads=32, hd=128)
    dyl = torch.randn(32768, 6144, device=dev).bfloat16()
    pre = torch.randn_like(dyl)
    dbl = torch.zeros(6144, device=dev)
    add("linear_bwd_prep_gelu", 3 * 2 * dyl.numel(),
        lambda: ext().linear_bwd_prep(dyl, pre, None, 32768, 1, dbl, True), rows=32768, N=6144)
    del dyl, pre
    n = 64 << 20
    p32, g32, m32, v32 = (torch.randn(n, device=dev) for _ in range(4))
    v32.abs_()
    p16 = torch.empty(n, device=dev, dtype=torch.bfloat16)
    sq = torch.ones(1, device=dev)
    add("adamw_flat", n * (4 * 4 + 3 * 4 + 2),
        lambda: ext().adamw_flat(p32, g32, m32, v32, p16, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1, 1.0, sq, 1.0), numel=n)
    return out


def bench_groupnorm(a) -> list[dict]:
    """VAE-decoder GroupNorm(32)+SiLU on channels-last [8, 128, 512, 512] bf16 (one read + one write pass
    after the statistics pass)."""
    from verl_omni_b200.ops.norm import group_norm_act

    x = torch.randn(8, 128, 512, 512, device="cuda").bfloat16().to(memory_format=torch.channels_last)
    w = torch.ones(128, device="cuda").bfloat16()
    b = torch.zeros(128, device="cuda").bfloat16()
    with torch.no_grad():
        ms = timeit(lambda: group_norm_act(x, w, b, 32, 1e-6, True), a.iters)
    nbytes = 3 * 2 * x.numel()  # stats read, apply read + write
    return [{"op": "group_norm_silu_nhwc", "shape": list(x.shape), "ms": round(ms, 4),
             "gbs": round(nbytes / ms / 1e6, 1)}]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "gemm_sweep", "gemm_pair", "ulysses", "tp", "fmha", "sde", "adaln", "optstep", "moe", "groupnorm", "decode", "rollout_decode", "rowops"])
    ap.add_argument("--numel", type=int, default=2_240_000_000)
    ap.add_argument("--M", type=int, default=21712)
    ap.add_argument("--N", type=int, default=6144)
    ap.add_argument("--K", type=int, default=1536)
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--H", type=int, default=24)
    ap.add_argument("--S", type=int, default=1357)
    ap.add_argument("--D", type=int, default=64)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--only", default="")
    ap.add_argument("--compare", action="store_true")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--new", type=int, default=64)
    a = ap.parse_args()
    pk = _peaks()
    rows = {"gemm": bench_gemm, "gemm_sweep": bench_gemm_sweep, "gemm_pair": bench_gemm_pair, "ulysses": bench_ulysses, "tp": bench_tp, "fmha": bench_fmha, "optstep": bench_optstep, "sde": bench_sde, "adaln": bench_adaln, "moe": bench_moe, "groupnorm": bench_groupnorm, "decode": bench_decode, "rollout_decode": bench_rollout_decode, "rowops": bench_rowops}[a.op](a)
    for r in rows:
        if "tflops" in r:
            r[f"frac_of_{pk['src']}_gemm_peak"] = round(r["tflops"] / pk["tflops"], 3)
        if "gbs" in r:
            r[f"frac_of_{pk['src']}_hbm"] = round(r["gbs"] / pk["gbs"], 3)
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
