"""torch.ops.cab.* without a GPU: the operators are registered on import, their fake
implementations give the output shapes and dtypes of the real ones, and a CPU tensor finds
no kernel (there is no CPU fallback)."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import cab_attention  # noqa: F401  (registers the operators)


def test_operators_registered():
    for name in ("coarsen_maxl2", "block_frc", "topk_blocks", "sparse_attn", "flash_attn"):
        assert hasattr(torch.ops.cab, name), name


def test_fake_shapes_follow_the_c_abi_outputs():
    B, Hq, Hkv, N, D, bs, k = 2, 8, 2, 1000, 128, 64, 3
    M = (N + bs - 1) // bs
    with FakeTensorMode():
        q = torch.empty(B, Hq, N, D, dtype=torch.bfloat16, device="cuda")
        kk = torch.empty(B, Hkv, N, D, dtype=torch.bfloat16, device="cuda")
        qc, kc, qi, ki = torch.ops.cab.coarsen_maxl2(q, kk, bs)
        assert qc.shape == (B, Hq, M, D) and kc.shape == (B, Hkv, M, D) and qc.dtype == torch.bfloat16
        assert qi.shape == (B, Hq, M) and ki.shape == (B, Hkv, M) and qi.dtype == torch.int32
        f = torch.ops.cab.block_frc(qc, kc, 1.0, 0.5, "additive", "abs", "none")
        assert f.shape == (B, Hq, M, M) and f.dtype == torch.float32
        idx, num = torch.ops.cab.topk_blocks(f, k, True, True, False)
        assert idx.shape == (B, Hq, M, k) and num.shape == (B, Hq, M) and idx.dtype == torch.int32
        o = torch.ops.cab.sparse_attn(q, kk, kk, idx, num, bs, False, 0.0)
        assert o.shape == q.shape and o.dtype == q.dtype
        o2, s = torch.ops.cab.flash_attn(q, kk, kk, True, 0.0, True)
        assert o2.shape == q.shape and s.shape == (B, Hq, N) and s.dtype == torch.float32


def test_cpu_tensors_find_no_kernel():
    x = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        torch.ops.cab.sparse_attn(x, x, x, torch.zeros(1, 1, 1, 1, dtype=torch.int32),
                                  torch.ones(1, 1, 1, dtype=torch.int32), 64, False, 0.0)
