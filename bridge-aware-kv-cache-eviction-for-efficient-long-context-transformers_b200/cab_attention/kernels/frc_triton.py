"""Node-level Forman-Ricci curvature of an attention graph (``cab_attention/kernels/
frc_triton.py`` of the reference, exported by its ``cab_attention/kernels/__init__.py``).

    F(i) = 4 w_i - 2 S_i + 3 T_i,   w_i = S_i = sum_j A_ij,   T_i = sum_j sum_k A_ij A_jk

All entry points run ``cab_node_frc`` (two HBM-bound passes: row sums, then
``T = A @ S``, since ``sum_k A_jk = S_j``) and return tensors in the input dtype like the
reference. ``compute_frc_pytorch`` (the reference's CPU-capable variant) and ``use_triton``
are kept for signature compatibility and run the same GPU kernel; there is no CPU path.
Inputs may carry leading batch dimensions ``[..., N, N]``.
"""

from __future__ import annotations

import torch

from .. import _lib


def _node_frc(attention: torch.Tensor):
    _lib.require_cuda(attention)
    if attention.dim() < 2 or attention.shape[-1] != attention.shape[-2]:
        raise ValueError("attention must be [..., N, N]")
    N = attention.shape[-1]
    lead = attention.shape[:-2]
    a = attention.contiguous()
    batch = a.numel() // (N * N) if N else 0
    frc = torch.empty(*lead, N, dtype=torch.float32, device=a.device)
    strengths = torch.empty_like(frc)
    triangles = torch.empty_like(frc)
    rc = _lib.lib().cab_node_frc(a.data_ptr(), frc.data_ptr(), strengths.data_ptr(), triangles.data_ptr(),
                                 batch, N, _lib.dtype_code(a), _lib.stream_of(a))
    _lib.check(rc, "cab_node_frc")
    dt = attention.dtype
    return frc.to(dt), strengths.to(dt), triangles.to(dt)


def compute_node_strengths_triton(attention: torch.Tensor) -> torch.Tensor:
    """Node strengths ``S_i = sum_j A_ij``."""
    return _node_frc(attention)[1]


def compute_triangles_triton(attention: torch.Tensor) -> torch.Tensor:
    """Weighted triangles ``T_i = sum_j sum_k A_ij A_jk``."""
    return _node_frc(attention)[2]


def compute_frc_triton(attention: torch.Tensor) -> torch.Tensor:
    """FRC per node: ``4 S - 2 S + 3 T`` (lower = bridge / bottleneck)."""
    return _node_frc(attention)[0]


def compute_frc_pytorch(attention: torch.Tensor) -> torch.Tensor:
    """Same result as ``compute_frc_triton`` (kept for signature compatibility)."""
    return _node_frc(attention)[0]


def compute_frc(attention: torch.Tensor, use_triton: bool = True) -> torch.Tensor:
    """FRC per node; ``use_triton`` is accepted and ignored (one implementation)."""
    return _node_frc(attention)[0]
