"""Prefill from host memory: the CAB path (coarsen -> FRC -> top-k -> block-sparse
attention) over page-locked CPU tensors, streamed through the GPU one (batch, KV head)
unit at a time so that the PCIe copies of neighbouring units overlap the compute
(``cab_prefill_host`` of the C ABI).

    out = prefill_from_host(q_pinned, k_pinned, v_pinned, sparsity=0.95)

Results equal ``CoarseCurvaturePredictor(...).predict_blocks(q, k)`` followed by
``block_sparse_attention`` on device copies of the same tensors, bit for bit. An addition
of this package: the reference's callers copy whole tensors with ``.to(device)`` /
``.cpu()`` around the layer (e.g. ``examples/demo_cab_attention.py:82,142``).
"""

from __future__ import annotations

import math

import torch

from . import _lib
from .kernels.frc_kernel import keep_count


def _pinned_cpu(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        raise ValueError(f"{name} must be a CPU tensor (device tensors: use the predictor and "
                         "block_sparse_attention directly)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if not t.is_pinned():
        raise ValueError(f"{name} must be in page-locked memory (tensor.pin_memory())")
    return t


@torch.no_grad()
def prefill_from_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, block_size: int = 64,
                      sparsity: float = 0.95, lambda_redundancy: float = 0.5,
                      temperature: float = 1.0, normalization: str = "abs",
                      formula: str = "additive", redundancy_scale: str = "none",
                      select_high: bool = True, keep_diagonal: bool = True, causal: bool = False,
                      softmax_scale: float | None = None, out: torch.Tensor | None = None,
                      return_indices: bool = False, device=None, synchronize: bool = True):
    """``q [B,Hq,N,D]``, ``k, v [B,Hkv,N,D]``: contiguous, pinned CPU tensors of one dtype.

    Returns ``out`` (pinned CPU, shaped like q; written in place when given) and, with
    ``return_indices``, the pinned CPU block lists ``kv_idx [B,Hq,M,keep]`` int32 and
    ``kv_num [B,Hq,M]`` int32. The predictor arguments and their defaults are those of
    ``CoarseCurvaturePredictor``. With ``synchronize=False`` the call returns once the work
    is queued on the device's current stream; the outputs are valid after that stream
    has been synchronised."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _pinned_cpu(name, t)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    if q.dim() != 4 or k.shape != v.shape or k.dim() != 4:
        raise ValueError("q must be [B, Hq, N, D] and k, v [B, Hkv, N, D]")
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if k.shape[0] != B or k.shape[2] != N or k.shape[3] != D or Hq % Hkv:
        raise ValueError("k and v must be [B, Hkv, N, D] with Hq % Hkv == 0")
    if not 0.0 <= sparsity < 1.0:
        raise ValueError("sparsity must be in [0, 1)")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    dummy = torch.empty(0, device=dev)
    _lib.require_cuda(dummy)
    M = (N + block_size - 1) // block_size
    keep = keep_count(M, sparsity)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    else:
        _pinned_cpu("out", out)
        if out.shape != q.shape or out.dtype != q.dtype:
            raise ValueError("out must match q's shape and dtype")
    kv_idx = kv_num = None
    if return_indices:
        kv_idx = torch.empty(B, Hq, M, keep, dtype=torch.int32).pin_memory()
        kv_num = torch.empty(B, Hq, M, dtype=torch.int32).pin_memory()
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    dt = _lib.dtype_code(q)
    norm = _lib.NORMALIZATIONS[normalization]
    L = _lib.lib()
    nbytes = _lib._c_size(0)
    with torch.cuda.device(dev):
        _lib.check(L.cab_prefill_host_workspace_size(B, Hq, Hkv, N, D, block_size, keep, dt, norm,
                                                     nbytes), "cab_prefill_host_workspace_size")
        ws = _lib.workspace(nbytes.value, dev)
        stream = torch.cuda.current_stream(dev)
        rc = L.cab_prefill_host(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                _lib.ptr(kv_idx), _lib.ptr(kv_num), B, Hq, Hkv, N, D, block_size,
                                keep, float(temperature), float(lambda_redundancy), norm,
                                _lib.FORMULAS[formula], _lib.REDUNDANCY_SCALES[redundancy_scale],
                                int(bool(select_high)), int(bool(keep_diagonal)),
                                int(bool(causal)), scale, dt, _lib.ptr(ws), nbytes.value,
                                stream.cuda_stream)
        _lib.check(rc, "cab_prefill_host")
        # The library's copy streams also touch `ws`, but the call joins them back into
        # `stream`, so the allocator's stream-ordered reuse of `ws` stays safe.
        if synchronize:
            stream.synchronize()
    return (out, kv_idx, kv_num) if return_indices else out
