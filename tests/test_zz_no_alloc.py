"""cab_sparse_attn_fwd_noalloc, the entry point for callers that cannot allocate device
memory (for example a host whose caching allocator owns the GPU's memory, or a binding
without a CUDA allocator): it must give the same attention output as the workspace entry
point cab_sparse_attn_fwd, call after call, using only the library's static scratch.

This file sorts last so that a run stopping at the first failure has already run every
other test; it also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

_lib = pytest.importorskip("cab_attention._lib")


def _noalloc(q, k, v, idx, num, out, lse, bs, causal):
    L = _lib.lib()
    B, Hq, N, D = q.shape
    rc = L.cab_sparse_attn_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), idx.data_ptr(), num.data_ptr(), out.data_ptr(),
        lse.data_ptr(), B, Hq, k.shape[1], N, D, bs, idx.shape[-1], _lib.strides3(q),
        _lib.strides3(k), _lib.strides3(v), _lib.strides3(out), 1.0 / D ** 0.5, int(causal),
        _lib.dtype_code(q), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.cab_last_error_string().decode()


def _case(seed, N, k, causal):
    from cab_attention.kernels import block_sparse_attention
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, D, bs = 1, 4, 2, 128, 64
    q = torch.randn(B, Hq, N, D, generator=g).to(torch.bfloat16).cuda()
    kk = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    M = (N + bs - 1) // bs
    F = torch.randn(B, Hq, M, M, generator=g).numpy()
    idx, num, _ = orc.topk_block_mask(F, k, True, True, causal)
    idx, num = torch.from_numpy(idx).cuda(), torch.from_numpy(num).cuda()
    want, wlse = block_sparse_attention(q, kk, v, idx, num, bs, causal, return_lse=True)
    out = torch.full_like(q, float("nan"))
    lse = torch.full((B, Hq, N), float("nan"), device="cuda")
    _noalloc(q, kk, v, idx, num, out, lse, bs, causal)
    torch.cuda.synchronize()
    return out, lse, want, wlse


def test_noalloc_matches_workspace_entry_point_twice():
    # two calls in a row with different shapes and lists: the second call must not see
    # anything the first one left in the shared scratch
    for seed, N, k, causal in ((1, 3000, 7, False), (2, 1800, 4, True)):
        out, lse, want, wlse = _case(seed, N, k, causal)
        assert torch.isfinite(out).all()
        assert (out.float() - want.float()).abs().max().item() <= 2e-2
        fin = torch.isfinite(wlse)
        assert torch.equal(torch.isfinite(lse), fin)
        assert (lse[fin] - wlse[fin]).abs().max().item() <= 2e-2
    assert _lib.device_status() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    # real device buffers of the rejected size, so that even if the size check regressed
    # the call would read and write memory it owns instead of a bad address
    L = _lib.lib()
    need = _lib._c_size(0)
    N, kmax, D = 1 << 20, 300, 128
    assert L.cab_sparse_attn_workspace_size(1, 1, N, D, 64, kmax, 2, ctypes.byref(need)) == 0
    assert need.value > (16 << 20)
    q = torch.zeros(1, 1, N, D, dtype=torch.bfloat16, device="cuda")
    k, v, out = torch.zeros_like(q), torch.zeros_like(q), torch.zeros_like(q)
    M = N // 64
    idx = torch.arange(kmax, dtype=torch.int32, device="cuda").repeat(M, 1).view(1, 1, M, kmax)
    num = torch.full((1, 1, M), kmax, dtype=torch.int32, device="cuda")
    lse = torch.zeros(1, 1, N, device="cuda")
    s = _lib._i64_3(N * D, N * D, D)
    rc = L.cab_sparse_attn_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), idx.data_ptr(),
                                       num.data_ptr(), out.data_ptr(), lse.data_ptr(), 1, 1, 1, N, D,
                                       64, kmax, s, s, s, s, 0.088, 0, 2,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert b"16 MiB" in L.cab_last_error_string()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
