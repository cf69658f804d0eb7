"""Block-sparse attention over the kept key blocks (the FlexAttention / manual
sparse-attention step of the reference's ``CABAttention``, ``README.md:44-46``;
manual path ``experiments/longbench_qa/methods.py:103-119,348-356``).

``block_sparse_attention(q, k, v, kv_idx, kv_num, block_size)``: for each query block i
of (b, h), softmax(q k^T * scale) v over the keys of blocks
``kv_idx[b, h, i, :kv_num[b, h, i]]`` of KV head h // (Hq // Hkv), -inf elsewhere (and
above the diagonal when ``causal``); a row without any key returns 0.
"""

from __future__ import annotations

import math

import torch

from .. import _lib


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_idx: torch.Tensor,
                           kv_num: torch.Tensor, block_size: int = 64, causal: bool = False,
                           softmax_scale: float | None = None, out: torch.Tensor | None = None,
                           return_lse: bool = False):
    """``q [B,Hq,N,D]``, ``k, v [B,Hkv,N,D]`` (strided views allowed: innermost dim dense,
    strides 16-byte aligned); ``kv_idx [B,Hq,M,kmax]`` int32 ascending, ``kv_num [B,Hq,M]``.
    Returns ``out`` shaped like q (or writes into the given ``out`` view); with
    ``return_lse`` also the natural-log sum-exp ``[B,Hq,N]`` fp32."""
    _lib.require_cuda(q, k, v, kv_idx, kv_num)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if k.shape != v.shape or k.shape[0] != B or k.shape[2] != N or k.shape[3] != D or Hq % Hkv:
        raise ValueError("k and v must be [B, Hkv, N, D] with Hq % Hkv == 0")
    M = (N + block_size - 1) // block_size
    if kv_idx.dim() != 4 or tuple(kv_idx.shape[:3]) != (B, Hq, M) or tuple(kv_num.shape) != (B, Hq, M):
        raise ValueError(f"kv_idx must be [B, Hq, {M}, kmax] and kv_num [B, Hq, {M}]")
    kv_idx = kv_idx.to(torch.int32).contiguous()
    kv_num = kv_num.to(torch.int32).contiguous()
    kmax = kv_idx.shape[3]

    def prep(t):
        if t.stride(3) != 1 or any((s * t.element_size()) % 16 for s in t.stride()[:3]) \
                or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    q, k, v = prep(q), prep(k), prep(v)
    if out is None:
        out = torch.empty(B, Hq, N, D, dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, Hq, N, D) or out.dtype != q.dtype or out.stride(3) != 1:
        raise ValueError("out must be [B, Hq, N, D] of q's dtype with a dense last dimension")
    lse = torch.empty(B, Hq, N, dtype=torch.float32, device=q.device) if return_lse else None
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    dt = _lib.dtype_code(q)
    L = _lib.lib()
    nbytes = _lib._c_size(0)
    _lib.check(L.cab_sparse_attn_workspace_size(B, Hq, N, D, block_size, kmax, dt, nbytes),
               "cab_sparse_attn_workspace_size")
    ws = _lib.workspace(nbytes.value, q.device)
    rc = L.cab_sparse_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_idx.data_ptr(),
                               kv_num.data_ptr(), out.data_ptr(), _lib.ptr(lse), B, Hq, Hkv, N, D,
                               block_size, kmax, _lib.strides3(q), _lib.strides3(k),
                               _lib.strides3(v), _lib.strides3(out), scale, int(bool(causal)), dt,
                               _lib.ptr(ws), nbytes.value, _lib.stream_of(q))
    _lib.check(rc, "cab_sparse_attn_fwd")
    return (out, lse) if return_lse else out


def sparse_attention_flops(kv_num: torch.Tensor, block_size: int, D: int) -> float:
    """Algorithmic FLOPs over kept block pairs: 4 * bs^2 * D per (query block, key block)."""
    return 4.0 * block_size * block_size * D * float(kv_num.sum().item())
