"""Allocation-free SDE-step entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory (an allocator callback, which would
re-enter the allocator; a host with a fixed memory budget; a plain C program without PyTorch's
allocator).  ``vo_sde_step_fwd_noalloc`` serves them with a fixed device array for its partial sums.
This test checks it against the allocating entry point on two consecutive calls.  The file name
makes pytest collect it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fn():
    from verl_omni_b200.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    f = lib.vo_sde_step_fwd_noalloc
    P = ctypes.c_void_p
    f.argtypes = [P, P, P, P, P, P, P, P, P, P, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                  ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, P]
    f.restype = ctypes.c_int
    return f


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("mode", ["seed", "prev", "noise"])
def test_noalloc_matches_allocating_entry_point(mode):
    from verl_omni_b200.ops._ext import ext

    f = _fn()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (B, shape, sde_type) in enumerate([(6, (16, 64, 64), 0), (3, (4, 40, 40), 2)]):
        torch.manual_seed(call)
        x = torch.randn(B, *shape, device="cuda")
        v = torch.randn(B, *shape, device="cuda")
        sig = torch.linspace(0.9, 0.2, B, device="cuda")
        sigp = sig - 0.1
        prev = torch.randn_like(x) if mode == "prev" else None
        noise = torch.randn_like(x) if mode == "noise" else None
        n = x[0].numel()
        ref_prev, ref_lp, ref_mean, ref_std = ext().sde_step_fwd(x, v, sig, sigp, prev, noise, 0.95, 0.7, sde_type,
                                                                 99 + call, 3, True, True)
        out_prev = torch.empty_like(x)
        mean = torch.empty_like(x)
        lp = torch.empty(B, device="cuda")
        std = torch.empty(B, device="cuda")
        rc = f(_ptr(x), _ptr(v), _ptr(sig), _ptr(sigp), _ptr(prev), _ptr(noise), _ptr(out_prev), _ptr(mean),
               _ptr(lp), _ptr(std), B, n, 0.95, 0.7, sde_type, 99 + call, 3, 1, 1, stream)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(mean, ref_mean, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(lp, ref_lp, rtol=1e-4, atol=1e-3)
        torch.testing.assert_close(std, ref_std, rtol=1e-5, atol=1e-6)
        if mode == "prev":
            # a distinct prev_out receives a copy of the caller's sample
            torch.testing.assert_close(out_prev, prev, rtol=0, atol=0)
        else:
            torch.testing.assert_close(out_prev, ref_prev, rtol=1e-4, atol=1e-4)


def test_noalloc_rejects_oversized_problem():
    f = _fn()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 100000 rows need at least 100000 partial-sum slots, more than the fixed scratch holds; every buffer
    # is still sized for the request so nothing could be touched out of bounds
    B, n = 100_000, 4
    x = torch.zeros(B, n, device="cuda")
    outs = [torch.empty(B, n, device="cuda") for _ in range(2)]
    sig = torch.full((B,), 0.5, device="cuda")
    vec = [torch.empty(B, device="cuda") for _ in range(2)]
    rc = f(_ptr(x), _ptr(x), _ptr(sig), _ptr(sig * 0.5), None, None, _ptr(outs[0]), _ptr(outs[1]), _ptr(vec[0]),
           _ptr(vec[1]), B, n, 0.95, 0.7, 0, 1, 0, 1, 1, stream)
    assert rc == -2


def test_noalloc_rejects_too_many_rows_for_the_grid():
    f = _fn()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 65536 rows with one chunk each fit the scratch but not the grid's row dimension
    B, n = 65536, 1
    x = torch.zeros(B, n, device="cuda")
    outs = [torch.empty(B, n, device="cuda") for _ in range(2)]
    sig = torch.full((B,), 0.5, device="cuda")
    vec = [torch.empty(B, device="cuda") for _ in range(2)]
    rc = f(_ptr(x), _ptr(x), _ptr(sig), _ptr(sig * 0.5), None, None, _ptr(outs[0]), _ptr(outs[1]), _ptr(vec[0]),
           _ptr(vec[1]), B, n, 0.95, 0.7, 0, 1, 0, 1, 1, stream)
    assert rc == -2
