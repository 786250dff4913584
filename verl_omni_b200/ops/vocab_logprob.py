"""log p(target) of a language-model head without a [tokens, vocab] fp32 logits tensor.

``token_logprobs_from_hidden(h, w, targets, temperature)`` equals
``log_softmax((h @ w.T).float() / T).gather(targets)`` (the reference computes it from full logits:
``verl_omni/workers/rollout/vllm_rollout/vllm_omni_async_server.py:537-579`` samples from them, and the
actor's log-prob recompute materialises them per micro-batch).  Here the vocabulary is processed in
chunks of ``chunk`` rows of ``w``: the tcgen05 GEMM writes one bf16 logits chunk, a row kernel folds it
into an online log-sum-exp and picks up the target logit (``csrc/vocab_logprob.cu``).  The backward
recomputes each chunk, turns it in place into ``dlogits = g / T (onehot - softmax)`` and runs the chunk's
dgrad GEMM and its weight-gradient GEMM (fp32, straight into ``w.main_grad`` when the engine owns one).
Peak extra memory: one ``[tokens, chunk]`` bf16 buffer.  CPU tensors take the same chunked path in fp32.
"""

from __future__ import annotations

import torch

from verl_omni_b200.ops import gemm as G

DEFAULT_CHUNK = 32768


def _logits_chunk(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if h.is_cuda:
        return G.linear_fwd(h, w, None)[0]
    return h.float() @ w.float().t()


class _ChunkedTokenLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, targets, temperature, chunk):
        N, V = h.shape[0], w.shape[0]
        inv_t = 1.0 / float(temperature)
        dev = h.device
        m = torch.full((N,), float("-inf"), device=dev)
        s = torch.zeros(N, device=dev)
        t = torch.zeros(N, device=dev)
        for lo in range(0, V, chunk):
            hi = min(V, lo + chunk)
            z = _logits_chunk(h, w[lo:hi])
            if h.is_cuda:
                from verl_omni_b200.ops._ext import ext

                ext().vocab_lse_update(z, lo, targets, inv_t, m, s, t)
            else:
                zf = z * inv_t
                mc = zf.max(-1).values
                mn = torch.maximum(m, mc)
                s = s * torch.exp(m - mn).nan_to_num(0.0) + torch.exp(zf - mn[:, None]).sum(-1)
                m = mn
                inside = (targets >= lo) & (targets < hi)
                idx = (targets - lo).clamp(0, hi - lo - 1)
                t = torch.where(inside, zf.gather(1, idx[:, None])[:, 0], t)
        lse = m + torch.log(s)
        ctx.save_for_backward(h, w, targets, lse)
        ctx.meta = (inv_t, chunk)
        return t - lse

    @staticmethod
    def backward(ctx, g):
        h, w, targets, lse = ctx.saved_tensors
        inv_t, chunk = ctx.meta
        g = g.float().contiguous()
        N, V = h.shape[0], w.shape[0]
        dh = torch.zeros(h.shape, device=h.device, dtype=torch.float32)
        mg = getattr(w, "main_grad", None)
        dw = None if (mg is not None or not ctx.needs_input_grad[1]) else torch.zeros(w.shape, device=w.device,
                                                                                        dtype=torch.float32)
        for lo in range(0, V, chunk):
            hi = min(V, lo + chunk)
            wc = w[lo:hi]
            z = _logits_chunk(h, wc)
            if h.is_cuda:
                from verl_omni_b200.ops._ext import ext

                ext().vocab_lse_grad(z, lo, targets, inv_t, lse, g)
                dz = z
            else:
                p = torch.exp(z * inv_t - lse[:, None])
                onehot = torch.zeros_like(p)
                inside = (targets >= lo) & (targets < hi)
                rows = torch.nonzero(inside)[:, 0]
                onehot[rows, targets[rows] - lo] = 1.0
                dz = (g[:, None] * inv_t) * (onehot - p)
            dh += G.matmul_nn(dz.to(h.dtype), wc).float() if h.is_cuda else dz @ wc.float()
            if mg is not None:
                G.wgrad(dz.to(h.dtype), h, mg[lo:hi]) if h.is_cuda else mg[lo:hi].add_(dz.t() @ h.float())
            elif dw is not None:
                dw[lo:hi] = G.wgrad(dz.to(h.dtype), h, None) if h.is_cuda else dz.t() @ h.float()
        return dh.to(h.dtype), (dw.to(w.dtype) if dw is not None else None), None, None, None


def token_logprobs_from_hidden(h: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0,
                               chunk: int = DEFAULT_CHUNK) -> torch.Tensor:
    """h [..., D] final hidden states, w [V, D] head weight, targets [...] ids -> fp32 log-probs [...]."""
    shape = targets.shape
    h2 = h.reshape(-1, h.shape[-1]).contiguous()
    out = _ChunkedTokenLogProb.apply(h2, w, targets.reshape(-1).to(torch.int64).contiguous(), float(temperature),
                                     int(chunk))
    return out.view(shape)
