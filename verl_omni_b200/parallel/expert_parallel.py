"""Expert parallelism: all-to-all token dispatch to expert-owning ranks and the inverse combine.

Each of ``ep`` ranks owns ``experts / ep`` consecutive experts.  For routed (token, slot) pairs the
dispatch sorts by destination rank, exchanges counts, then rows with a variable-size all-to-all; the
owners run their experts on the received rows; the combine sends results back along the same split
sizes and adds them into the token outputs weighted by the router gates.  Both exchanges are autograd
functions (backward = the opposite exchange with swapped splits).  NCCL uses ``all_to_all_single``
with split sizes; gloo ranks emulate it with an all-gather of padded chunks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from verl_omni_b200.parallel import dist as D


def all_to_all_v(x: torch.Tensor, send: list[int], recv: list[int], group) -> torch.Tensor:
    ws = D.world_size(group)
    if ws == 1:
        return x
    out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
    if dist.get_backend(group) == "nccl":
        dist.all_to_all_single(out, x.contiguous(), output_split_sizes=recv, input_split_sizes=send, group=group)
        return out
    mt = torch.tensor([max(max(send), max(recv), 1)], dtype=torch.int64)
    dist.all_reduce(mt, op=dist.ReduceOp.MAX, group=group)  # gloo all_gather needs equal sizes everywhere
    m = int(mt.item())
    chunks = list(x.split(send, 0))
    padded = torch.stack([torch.cat([c, c.new_zeros((m - c.shape[0],) + tuple(c.shape[1:]))]) for c in chunks])
    parts = [torch.empty_like(padded) for _ in range(ws)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    me = D.rank(group)
    return torch.cat([parts[src][me][: recv[src]] for src in range(ws)], 0)


class _A2AV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send, recv, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        return all_to_all_v(x, send, recv, group)

    @staticmethod
    def backward(ctx, g):
        return all_to_all_v(g.contiguous(), ctx.recv, ctx.send, ctx.group), None, None, None


class ExpertParallel:
    def __init__(self, num_experts: int, group=None):
        self.group = group
        self.ep = D.world_size(group)
        self.rank = D.rank(group)
        if num_experts % self.ep:
            raise ValueError(f"{num_experts} experts do not split over EP={self.ep}")
        self.per_rank = num_experts // self.ep
        self.local_experts = range(self.rank * self.per_rank, (self.rank + 1) * self.per_rank)

    def dispatch_combine(self, h: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor, expert_fn) -> torch.Tensor:
        T, K = idx.shape
        flat_e = idx.reshape(-1)
        tok = torch.arange(T, device=h.device).repeat_interleave(K)
        dest = flat_e // self.per_rank
        order = torch.argsort(dest * (self.per_rank * self.ep) + flat_e, stable=True)
        send_counts = torch.bincount(dest, minlength=self.ep)
        recv_counts = send_counts.clone()
        if self.ep > 1:
            recv_counts = torch.empty_like(send_counts)
            if dist.get_backend(self.group) == "nccl":
                dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            else:
                allc = [torch.empty_like(send_counts) for _ in range(self.ep)]
                dist.all_gather(allc, send_counts, group=self.group)
                recv_counts = torch.stack([allc[s][self.rank] for s in range(self.ep)])
        send, recv = send_counts.tolist(), recv_counts.tolist()
        x_send = h.index_select(0, tok[order])
        e_send = flat_e[order]
        x_recv = _A2AV.apply(x_send, send, recv, self.group)
        e_recv = all_to_all_v(e_send[:, None], send, recv, self.group)[:, 0]
        # experts process their rows grouped by expert id
        o = torch.argsort(e_recv, stable=True)
        y_sorted = expert_fn(x_recv.index_select(0, o), e_recv[o])
        y = torch.empty_like(y_sorted).index_copy(0, o, y_sorted)
        y_back = _A2AV.apply(y, recv, send, self.group)
        w = gates.reshape(-1)[order].unsqueeze(-1).to(y_back.dtype)
        out = torch.zeros_like(h)
        return out.index_add(0, tok[order], y_back * w)


    def decode_combine(self, h: torch.Tensor, idx: torch.Tensor, gates: torch.Tensor, w_gate_up, w_down,
                       e0: int) -> torch.Tensor:
        """Expert layer for a gradient-free step of a few tokens per rank (decode): every rank's tokens, expert
        ids and gates are all-gathered (one packed buffer), each rank applies its own experts to all of them,
        and a reduce-scatter sums the contributions back to the tokens' owners.  Every message has a fixed size,
        so nothing waits on the host (the variable all-to-all reads its split sizes on the host every layer).
        All ranks must call it with the same token count."""
        from verl_omni_b200.ops import moe as MO

        T, K = idx.shape
        Dm = h.shape[1]
        W = self.ep
        # idx travels as bf16: expert ids < 256 are exact
        pack = torch.cat([h.to(torch.bfloat16), gates.to(torch.bfloat16), idx.to(torch.bfloat16)], 1)
        allp = torch.empty(W * T, pack.shape[1], dtype=pack.dtype, device=h.device)
        D.all_gather_into(allp.view(-1), pack.contiguous().view(-1), self.group)
        hg = allp[:, :Dm].contiguous()
        gg = allp[:, Dm:Dm + K].float()
        ig = allp[:, Dm + K:].float().round().to(torch.int64)
        if MO.native_ok(hg, w_gate_up, w_down):
            part = MO.moe_ffn_local(hg, ig, gg, w_gate_up, w_down, e0)
        else:
            part = MO.moe_ffn_local_reference(hg, ig, gg, w_gate_up, w_down, e0)
        out = torch.empty(T, Dm, dtype=torch.float32, device=h.device)
        D.reduce_scatter_into(out.view(-1), part.contiguous().view(-1), self.group)
        return out.to(h.dtype)


# ---------------------------------------------------------------- fused exchange over peer memory
class _Layout:
    """Host plan of one fused exchange (computed from the all-gathered per-expert counts)."""

    def __init__(self, C, rank: int, El: int):
        import numpy as np

        W, E = C.shape
        self.total = C.sum(0)                                   # rows per expert over all sources
        self.padded = (self.total + 127) // 128 * 128
        blk = self.padded.reshape(W, El)
        self.seg_start = (np.cumsum(blk, 1) - blk).reshape(E)    # within the owner's buffer
        self.rows = blk.sum(1)                                   # padded rows per owner
        self.src_prefix = np.cumsum(C, 0) - C                    # [W, E]: rows of lower source ranks
        self.first = np.cumsum(C, 1) - C                         # [W, E]: slot of an expert's first pair per source
        self.P = C.sum(1)                                        # pairs per source
        r, lo, hi = rank, rank * El, (rank + 1) * El
        # this rank's owned rows: expert j, source s, i-th pair -> (source rank s, slot first[s, e] + i)
        ranks, slots, rows = [], [], []
        for e in range(lo, hi):
            for s in range(W):
                n = int(C[s, e])
                if n:
                    rows.append(self.seg_start[e] + self.src_prefix[s, e] + np.arange(n))
                    ranks.append(np.full(n, s, dtype=np.int32))
                    slots.append(self.first[s, e] + np.arange(n))
        cat = lambda xs, dt: np.concatenate(xs).astype(dt) if xs else np.zeros(0, dt)  # noqa: E731
        self.own_rows, self.own_rank, self.own_slot = cat(rows, np.int64), cat(ranks, np.int32), cat(slots, np.int64)
        pad = [self.seg_start[e] + self.total[e] + np.arange(self.padded[e] - self.total[e]) for e in range(lo, hi)]
        self.pad_rows = cat(pad, np.int64)
        R = int(self.rows[r])
        self.R = R
        local_pad = self.padded[lo:hi]
        self.seg_local = np.concatenate([[0], np.cumsum(local_pad)]).astype(np.int32)
        self.tile_expert = np.repeat(np.arange(El, dtype=np.int32), local_pad // 128)


class _FusedEP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, gates, w_gate_up, w_down, idx, ep):
        import numpy as np

        from verl_omni_b200.ops._ext import ext

        e_ = ext()
        dev = h.device
        T, K = idx.shape
        E, D = ep.per_rank * ep.ep, h.shape[1]
        W, r, El = ep.ep, ep.rank, ep.per_rank
        flat_e = idx.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        sorted_e = flat_e[order]
        tok_s = torch.arange(T, device=dev).repeat_interleave(K)[order]
        cnt = torch.bincount(flat_e, minlength=E).to(torch.int64)
        C_all = torch.empty(W, E, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(C_all, cnt, group=ep.group)
        C = C_all.cpu().numpy()  # one small host read per layer: buffer sizes and row maps
        L = _Layout(C, r, El)
        cap = int(-(-int(L.rows.max()) // 4096) * 4096) or 4096
        pcap = int(-(-int(L.P.max()) // 1024) * 1024) or 1024
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt, non_blocking=True)  # noqa: E731
        seg_start, src_prefix, first = (t(L.seg_start, torch.int64), t(L.src_prefix[r], torch.int64),
                                        t(L.first[r], torch.int64))
        dst_rank = (sorted_e // El).to(torch.int32)
        dst_row = seg_start[sorted_e] + src_prefix[sorted_e] + (torch.arange(order.numel(), device=dev) - first[sorted_e])
        plan = {"dst_rank": dst_rank, "dst_row": dst_row, "own_rows": t(L.own_rows, torch.int64),
                "own_rank": t(L.own_rank, torch.int32), "own_slot": t(L.own_slot, torch.int64),
                "pad_rows": t(L.pad_rows, torch.int64), "tile": t(L.tile_expert, torch.int32),
                "seg": t(L.seg_local, torch.int32), "R": L.R, "cap": cap, "pcap": pcap}
        # dispatch: every routed row straight into its owner's padded expert-sorted buffer
        xd = ep.buf("x", cap * D, dev)
        xv = xd.tensor.view(cap, D)
        if plan["pad_rows"].numel():
            xv.index_fill_(0, plan["pad_rows"], 0)
        e_.peer_row_copy(h.contiguous(), tok_s, dst_rank, dst_row, xd.peer_ptrs, cap)
        ep.barrier(dev)
        R = L.R
        wgu_l, wd_l = _local(w_gate_up, r, El), _local(w_down, r, El)
        x_own = xv[:R].clone()
        if R:
            gu = e_.moe_gemm_fwd(x_own, wgu_l, plan["tile"])
            a = e_.swiglu_fwd(gu)
            y = e_.moe_gemm_fwd(a, wd_l, plan["tile"])
        else:
            gu = a = y = h.new_zeros(0, D)
        # combine: every expert output row back to the slot of the rank that routed it
        yc = ep.buf("y", pcap * D, dev)
        if R:
            e_.peer_row_copy(y, plan["own_rows"], plan["own_rank"], plan["own_slot"], yc.peer_ptrs, pcap)
        ep.barrier(dev)
        P = order.numel()
        ys = yc.tensor.view(pcap, D)[:P].clone()
        gs = gates.reshape(-1)[order]
        out = torch.zeros_like(h).index_add(0, tok_s, (ys.float() * gs.float()[:, None]).to(h.dtype))
        ctx.save_for_backward(ys, gs, x_own, gu, a, w_gate_up, w_down)
        ctx.plan, ctx.ep, ctx.order, ctx.tok_s, ctx.shape = plan, ep, order, tok_s, (T, K)
        return out

    @staticmethod
    def backward(ctx, dout):
        from verl_omni_b200.ops._ext import ext

        e_ = ext()
        ys, gs, x_own, gu, a, w_gate_up, w_down = ctx.saved_tensors
        plan, ep, order, tok_s = ctx.plan, ctx.ep, ctx.order, ctx.tok_s
        T, K = ctx.shape
        dev = dout.device
        D = dout.shape[1]
        El, r = ep.per_rank, ep.rank
        dys = dout.contiguous()[tok_s]
        dg_sorted = (dys.float() * ys.float()).sum(-1)
        dy_slot = (dys.float() * gs.float()[:, None]).to(dout.dtype)
        dgates = torch.zeros(order.numel(), device=dev, dtype=torch.float32).index_copy(0, order, dg_sorted)
        # output gradients to the expert owners (same rows as the dispatch)
        cap, pcap, R = plan["cap"], plan["pcap"], plan["R"]
        db = ep.buf("x", cap * D, dev)
        dv = db.tensor.view(cap, D)
        if plan["pad_rows"].numel():
            dv.index_fill_(0, plan["pad_rows"], 0)
        e_.peer_row_copy(dy_slot, torch.arange(order.numel(), device=dev), plan["dst_rank"], plan["dst_row"],
                         db.peer_ptrs, cap)
        ep.barrier(dev)
        # weight gradients go straight into the (local) experts' fp32 main_grad when the engine owns one
        mg_gu, mg_d = getattr(w_gate_up, "main_grad", None), getattr(w_down, "main_grad", None)
        gwgu = mg_gu if mg_gu is not None else torch.zeros(w_gate_up.shape, device=dev, dtype=torch.float32)
        gwd = mg_d if mg_d is not None else torch.zeros(w_down.shape, device=dev, dtype=torch.float32)
        wgu_l, wd_l = _local(w_gate_up, r, El), _local(w_down, r, El)
        if R:
            dyo = dv[:R].clone()
            da = e_.moe_gemm_dgrad(dyo, wd_l, plan["tile"])
            e_.moe_gemm_wgrad(dyo, a, plan["seg"], _local(gwd, r, El), True)
            dgu = e_.swiglu_bwd(da, gu)
            dx = e_.moe_gemm_dgrad(dgu, wgu_l, plan["tile"])
            e_.moe_gemm_wgrad(dgu, x_own, plan["seg"], _local(gwgu, r, El), True)
        xb = ep.buf("y", pcap * D, dev)
        if R:
            e_.peer_row_copy(dx, plan["own_rows"], plan["own_rank"], plan["own_slot"], xb.peer_ptrs, pcap)
        ep.barrier(dev)
        dxs = xb.tensor.view(pcap, D)[:order.numel()]
        dh = torch.zeros(T, D, device=dev, dtype=dout.dtype).index_add(0, tok_s, dxs)
        return (dh, dgates.view(T, K).to(dout.dtype), None if mg_gu is not None else gwgu.to(w_gate_up.dtype),
                None if mg_d is not None else gwd.to(w_down.dtype), None, None)


def _local(w: torch.Tensor, r: int, El: int) -> torch.Tensor:
    """This rank's experts of a stacked expert tensor: the whole tensor when it holds only the local experts
    (expert-sharded model), else slice [r El, (r + 1) El)."""
    return w if w.shape[0] == El else w[r * El:(r + 1) * El]


class FusedExpertParallel(ExpertParallel):
    """Expert parallelism whose dispatch and combine are row copies into the peers' symmetric buffers
    (``csrc/ep.cu``), around the expert-grouped GEMMs of each owner: every routed row lands directly in its
    owner's expert-sorted, 128-row-padded GEMM input, and every output row directly in the slot of the rank
    that routed it -- no NCCL all-to-all, no host-side split sizes in the exchange (one small all-gather of
    the per-expert counts sizes the buffers).  Buffers are symmetric pairs used alternately, each use between
    one-element all-reduces."""

    def __init__(self, num_experts: int, group=None):
        super().__init__(num_experts, group)
        self._pairs: dict = {}

    def buf(self, key: str, numel: int, device):
        from verl_omni_b200.parallel.symm_mem import SymmetricBuffer

        k = (key, numel)
        if k not in self._pairs:
            self._pairs[k] = [[SymmetricBuffer(numel, torch.bfloat16, device, self.group) for _ in range(2)], 0]
        bufs, i = self._pairs[k]
        self._pairs[k][1] ^= 1
        return bufs[i]

    def barrier(self, device) -> None:
        from verl_omni_b200.parallel.symm_mem import stream_barrier

        stream_barrier(self.group, device)

    def fused_ok(self, h: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> bool:
        from verl_omni_b200.ops import moe as MO
        from verl_omni_b200.parallel.symm_mem import available

        if not (MO.native_ok(h, w_gate_up, w_down) and self.ep <= 8 and hasattr(_ext_mod(), "peer_row_copy")):
            return False
        if not hasattr(self, "_avail"):
            self._avail = available(self.group)
        return self._avail

    def dispatch_combine_fused(self, h, idx, gates, w_gate_up, w_down) -> torch.Tensor:
        return _FusedEP.apply(h, gates, w_gate_up, w_down, idx, self)

    def release(self) -> None:
        for bufs, _ in self._pairs.values():
            for b in bufs:
                b.close()
        self._pairs.clear()


def _ext_mod():
    from verl_omni_b200.ops._ext import ext

    return ext()
