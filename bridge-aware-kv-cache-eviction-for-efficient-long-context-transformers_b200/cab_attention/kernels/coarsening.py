"""Max-L2 block coarsening (``cab_attention/kernels/coarsening.py`` of the reference).

The reference exposes ``coarsen_qk_max_l2`` (Triton) and ``coarsen_qk_max_l2_pytorch``
(called by ``benchmarks/kernel_benchmark.py:82-85``, ``benchmarks/quick_kernel_test.py:54-57``
and ``experiments/longbench_qa/methods.py:303,327``); both names return
``(q_coarse, k_coarse)`` of shape ``[B, H, M, D]``, M = ceil(N / block_size), holding the
token of each block with the largest L2 norm (``README.md:30-32``). Here both names run
the sm_100a kernel ``cab_coarsen_maxl2``: norms are accumulated in fp64, the lowest
index wins ties, and a partial last block uses its valid tokens.
"""

from __future__ import annotations

import torch

from .. import _lib


def _coarsen(q, k, block_size, return_indices):
    ts = [t for t in (q, k) if t is not None]
    if not ts:
        raise ValueError("nothing to coarsen")
    _lib.require_cuda(*ts)
    dtype = ts[0].dtype
    if any(t.dtype != dtype for t in ts):
        raise TypeError("q and k must share a dtype")
    B, _, N, D = ts[0].shape
    Hq = q.shape[1] if q is not None else 0
    Hkv = k.shape[1] if k is not None else 0
    for t in ts:
        if t.dim() != 4 or t.shape[0] != B or t.shape[2] != N or t.shape[3] != D:
            raise ValueError("q and k must be [B, H, N, D] with matching B, N, D")
    M = (N + block_size - 1) // block_size
    dev = ts[0].device

    def prep(t):
        if t is None:
            return None
        if t.stride(3) != 1 or any((s * t.element_size()) % 16 for s in t.stride()[:3]) \
                or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    q, k = prep(q), prep(k)
    qc = torch.empty(B, Hq, M, D, dtype=dtype, device=dev) if q is not None else None
    kc = torch.empty(B, Hkv, M, D, dtype=dtype, device=dev) if k is not None else None
    qi = torch.empty(B, Hq, M, dtype=torch.int32, device=dev) if (q is not None and return_indices) else None
    ki = torch.empty(B, Hkv, M, dtype=torch.int32, device=dev) if (k is not None and return_indices) else None
    rc = _lib.lib().cab_coarsen_maxl2(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(qc), _lib.ptr(kc), _lib.ptr(qi), _lib.ptr(ki),
        B, Hq, Hkv, N, D, block_size,
        _lib.strides3(q) if q is not None else None,
        _lib.strides3(k) if k is not None else None,
        _lib.dtype_code(ts[0]), _lib.stream_of(ts[0]))
    _lib.check(rc, "cab_coarsen_maxl2")
    return qc, kc, qi, ki


def coarsen_qk_max_l2(q: torch.Tensor, k: torch.Tensor, block_size: int = 64,
                      return_indices: bool = False):
    """``(q_coarse, k_coarse)`` by Max-L2 pooling; with ``return_indices`` also the int32
    absolute token indices ``(q_idx, k_idx)`` of the chosen tokens.

    ``q [B,Hq,N,D]`` and ``k [B,Hkv,N,D]`` may be strided views (innermost dimension dense,
    16-byte aligned strides), e.g. heads sliced out of a fused QKV projection.
    """
    qc, kc, qi, ki = _coarsen(q, k, int(block_size), return_indices)
    if return_indices:
        return qc, kc, qi, ki
    return qc, kc


def coarsen_qk_max_l2_pytorch(q: torch.Tensor, k: torch.Tensor, block_size: int = 64):
    """The reference's PyTorch-named entry point; runs the same sm_100a kernel."""
    return coarsen_qk_max_l2(q, k, block_size)


def coarsen_max_l2(x: torch.Tensor, block_size: int = 64, return_indices: bool = False):
    """Max-L2 coarsening of one ``[B,H,N,D]`` tensor."""
    xc, _, xi, _ = _coarsen(x, None, int(block_size), return_indices)
    return (xc, xi) if return_indices else xc
