"""Paged KV cache block manager: allocation, reuse after a sequence frees its blocks, and decode attention
through the block table equal to the contiguous cache."""

import pytest
import torch

from verl_omni_b200.ops.decode import KVCache, PagedKVCache, decode_attention


def test_paged_cache_matches_contiguous_and_reuses_blocks():
    torch.manual_seed(0)
    pc = PagedKVCache(16, 2, 8, 64, "cpu", torch.float32)
    kc = KVCache(2, 2, 64, 64, "cpu", torch.float32)
    tmp = pc.add_sequence()
    pc.append([tmp], torch.randn(1, 2, 20, 64), torch.randn(1, 2, 20, 64))  # 3 blocks
    sids = [pc.add_sequence(), pc.add_sequence()]
    for n in (11, 1, 1, 9):
        if n == 1 and tmp is not None:
            pc.free_sequence(tmp)  # its blocks go back to the free list and are reused below
            tmp = None
        k, v = torch.randn(2, 2, n, 64), torch.randn(2, 2, n, 64)
        pc.append(sids, k, v)
        kc.append(k, v)
    table = pc.block_table(sids)
    assert set(table.flatten().tolist()) & {0, 1, 2}  # freed blocks were handed out again
    q = torch.randn(2, 4, 64)
    a = decode_attention(q, pc.k, pc.v, pc.lens(sids), block_table=table)
    b = decode_attention(q, kc.k, kc.v, kc.lens())
    torch.testing.assert_close(a, b)


def test_paged_cache_out_of_blocks():
    pc = PagedKVCache(2, 1, 4, 64, "cpu", torch.float32)
    s = pc.add_sequence()
    pc.append([s], torch.randn(1, 1, 8, 64), torch.randn(1, 1, 8, 64))
    with pytest.raises(RuntimeError, match="out of blocks"):
        pc.append([s], torch.randn(1, 1, 1, 64), torch.randn(1, 1, 1, 64))
