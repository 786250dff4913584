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
