"""Coarse Forman-Ricci score and block-mask generation
(``cab_attention/kernels/frc_kernel.py`` of the reference).

* ``compute_block_frc(q_coarse, k_coarse, temperature, lambda_redundancy, formula,
  normalization)`` -> ``(frc, affinity, redundancy)``, each ``[B, Hq, M, M]`` fp32
  (callers ``experiments/longbench_qa/methods.py:330-336``, ``benchmarks/kernel_benchmark.py:149``).
* ``generate_block_mask(frc, sparsity, select_high, keep_diagonal, causal, ...)`` -> bool
  ``[B, H, M, M]`` (callers ``methods.py:339-345``, ``kernel_benchmark.py:197-205``).
* ``visualize_frc_statistics(frc, affinity, triangles)`` (``README.md:106-111``).

Definitions (one set of flags, defaults named):
  A = Qc Kc^T / sqrt(D) / temperature;  Direct = |A| ("abs", default) | min-max | A ("raw");
  T = Direct @ Direct (``redundancy_scale="inv_m"``: / M);
  F = Direct - lambda T ("additive", default) | Direct / (1 + lambda T / (Direct + 1e-8))
  ("multiplicative"). ``affinity`` returned = Direct, ``redundancy`` = T.
Mask: per (b, h, row) keep k = max(1, int(M * (1 - sparsity))) blocks, the highest F when
``select_high`` (default, as passed by ``methods.py:342``) else the lowest; ties go to
the lower block index; ``keep_diagonal`` forces block i; ``causal`` restricts row i to
j <= i and keeps min(k, i + 1).
"""

from __future__ import annotations

import math

import torch

from .. import _lib


def keep_count(num_blocks: int, sparsity: float) -> int:
    """Blocks kept per row, ``max(1, int(M * (1 - sparsity)))`` (methods.py:252)."""
    return max(1, int(num_blocks * (1.0 - sparsity)))


def compute_block_frc(q_coarse: torch.Tensor, k_coarse: torch.Tensor, temperature: float = 1.0,
                      lambda_redundancy: float = 0.5, formula: str = "additive",
                      normalization: str = "abs", redundancy_scale: str = "none",
                      return_affinity: bool = True, return_redundancy: bool = True):
    """Coarse FRC on the tensor cores -> ``(frc, affinity, redundancy)``.

    ``q_coarse [B,Hq,M,D]``, ``k_coarse [B,Hkv,M,D]`` (Hq a multiple of Hkv; query head h
    uses KV head h // (Hq // Hkv)). ``return_affinity`` / ``return_redundancy`` = False
    skip those outputs (returned as None) and their HBM writes.
    """
    _lib.require_cuda(q_coarse, k_coarse)
    if formula not in _lib.FORMULAS:
        raise ValueError(f"formula must be one of {sorted(_lib.FORMULAS)}")
    if normalization not in _lib.NORMALIZATIONS:
        raise ValueError(f"normalization must be one of {sorted(_lib.NORMALIZATIONS)}")
    if redundancy_scale not in _lib.REDUNDANCY_SCALES:
        raise ValueError(f"redundancy_scale must be one of {sorted(_lib.REDUNDANCY_SCALES)}")
    if q_coarse.dtype != k_coarse.dtype:
        raise TypeError("q_coarse and k_coarse must share a dtype")
    B, Hq, M, D = q_coarse.shape
    Hkv = k_coarse.shape[1]
    if k_coarse.shape[0] != B or k_coarse.shape[2] != M or k_coarse.shape[3] != D or Hq % Hkv:
        raise ValueError("k_coarse must be [B, Hkv, M, D] with Hq % Hkv == 0")
    qc, kc = q_coarse.contiguous(), k_coarse.contiguous()
    dev = qc.device
    frc = torch.empty(B, Hq, M, M, dtype=torch.float32, device=dev)
    aff = torch.empty_like(frc) if return_affinity else None
    red = torch.empty_like(frc) if return_redundancy else None
    dt = _lib.dtype_code(qc)
    norm = _lib.NORMALIZATIONS[normalization]
    L = _lib.lib()
    nbytes = _lib._c_size(0)
    _lib.check(L.cab_frc_workspace_size(B, Hq, M, D, dt, norm, nbytes), "cab_frc_workspace_size")
    ws = _lib.workspace(nbytes.value, dev)
    rc = L.cab_frc(qc.data_ptr(), kc.data_ptr(), frc.data_ptr(), _lib.ptr(aff), _lib.ptr(red),
                   B, Hq, Hkv, M, D, dt, float(temperature), float(lambda_redundancy), norm,
                   _lib.FORMULAS[formula], _lib.REDUNDANCY_SCALES[redundancy_scale],
                   _lib.ptr(ws), nbytes.value, _lib.stream_of(qc))
    _lib.check(rc, "cab_frc")
    return frc, aff, red


def topk_blocks(scores: torch.Tensor, k: int, select_high: bool = True, keep_diagonal: bool = True,
                causal: bool = False, return_dense: bool = True,
                magnitude_scores: torch.Tensor | None = None, magnitude_ratio: float = 0.5):
    """Per-row top-k -> ``(kv_idx [B,H,M,k] int32 ascending, -1 padded; kv_num [B,H,M] int32;
    dense bool [B,H,M,M] or None)``. With ``magnitude_scores`` (same shape) the budget is
    split as in ``generate_block_mask``'s hybrid mode."""
    _lib.require_cuda(scores, magnitude_scores)
    if scores.dtype != torch.float32:
        scores = scores.float()
    scores = scores.contiguous()
    B, H, M, M2 = scores.shape
    if M != M2:
        raise ValueError("scores must be [B, H, M, M]")
    k = int(k)
    if not 1 <= k <= M:
        raise ValueError(f"k={k} outside [1, {M}]")
    dev = scores.device
    kv_idx = torch.empty(B, H, M, k, dtype=torch.int32, device=dev)
    kv_num = torch.empty(B, H, M, dtype=torch.int32, device=dev)
    dense = torch.empty(B, H, M, M, dtype=torch.bool, device=dev) if return_dense else None
    L = _lib.lib()
    if magnitude_scores is None:
        rc = L.cab_topk_blocks(scores.data_ptr(), kv_idx.data_ptr(), kv_num.data_ptr(), _lib.ptr(dense),
                               B * H, M, k, int(bool(select_high)), int(bool(keep_diagonal)),
                               int(bool(causal)), _lib.stream_of(scores))
        _lib.check(rc, "cab_topk_blocks")
    else:
        if tuple(magnitude_scores.shape) != (B, H, M, M):
            raise ValueError("magnitude_scores must have the shape of the FRC scores")
        if not 0.0 <= float(magnitude_ratio) <= 1.0:
            raise ValueError("magnitude_ratio must be in [0, 1]")
        mag = magnitude_scores.float().contiguous()
        rc = L.cab_topk_blocks_hybrid(scores.data_ptr(), mag.data_ptr(), kv_idx.data_ptr(),
                                      kv_num.data_ptr(), _lib.ptr(dense), B * H, M, k,
                                      float(magnitude_ratio), int(bool(select_high)),
                                      int(bool(keep_diagonal)), int(bool(causal)), _lib.stream_of(scores))
        _lib.check(rc, "cab_topk_blocks_hybrid")
    return kv_idx, kv_num, dense


def generate_block_mask(frc_scores: torch.Tensor, sparsity: float = 0.95, select_high: bool = True,
                        keep_diagonal: bool = True, causal: bool = False,
                        magnitude_scores: torch.Tensor | None = None, magnitude_ratio: float = 0.5,
                        return_indices: bool = False):
    """Dense bool block mask ``[B,H,M,M]`` (True = keep); with ``return_indices`` also
    ``(kv_idx, kv_num)`` for ``block_sparse_attention``.

    Hybrid (CAB V4, ``magnitude_scores`` given): per row, after the forced diagonal,
    ``int(r * magnitude_ratio)`` of the remaining budget ``r`` go to the largest magnitude
    scores and the rest to the best FRC scores among the blocks not yet taken
    (``experiments/longbench_qa/methods.py:407-418``: "reserve X% of budget for
    top-magnitude blocks, (1-X)% for top-FRC blocks")."""
    M = frc_scores.shape[-1]
    kv_idx, kv_num, dense = topk_blocks(frc_scores, keep_count(M, sparsity), select_high,
                                        keep_diagonal, causal, return_dense=True,
                                        magnitude_scores=magnitude_scores,
                                        magnitude_ratio=magnitude_ratio)
    if return_indices:
        return dense, kv_idx, kv_num
    return dense


def block_max_pool(attention_weights: torch.Tensor, block_size: int = 64) -> torch.Tensor:
    """Block-level magnitude scores of a dense attention matrix ``[B,H,N,N]``: the maximum
    of each ``block_size`` x ``block_size`` tile (zero padding of a partial block included),
    ``[B,H,M,M]`` in the input dtype (``CABV4Attention._coarsen_attention``,
    ``experiments/longbench_qa/methods.py:535-553``)."""
    _lib.require_cuda(attention_weights)
    B, H, N, N2 = attention_weights.shape
    if N != N2:
        raise ValueError("attention_weights must be [B, H, N, N]")
    a = attention_weights.contiguous()
    M = (N + block_size - 1) // block_size
    out = torch.empty(B, H, M, M, dtype=torch.float32, device=a.device)
    rc = _lib.lib().cab_block_maxpool(a.data_ptr(), out.data_ptr(), B * H, N, block_size,
                                      _lib.dtype_code(a), _lib.stream_of(a))
    _lib.check(rc, "cab_block_maxpool")
    return out.to(attention_weights.dtype)


def visualize_frc_statistics(frc_scores, affinity=None, triangles=None, save_path=None):
    """Summary statistics of the FRC / affinity / triangle matrices.

    Returns a dict; when matplotlib is importable and ``save_path`` is given, also writes
    histograms there (headless ``Agg`` backend).
    """
    stats = {}
    for name, t in (("frc", frc_scores), ("affinity", affinity), ("triangles", triangles)):
        if t is None:
            continue
        x = t.detach().float()
        stats[name] = {"mean": x.mean().item(), "std": x.std().item(), "min": x.min().item(),
                       "max": x.max().item(), "negative_fraction": (x < 0).float().mean().item()}
    if save_path is not None:
        try:
            import matplotlib
            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError:
            return stats
        fig, axes = plt.subplots(1, len(stats), figsize=(6 * len(stats), 4))
        axes = [axes] if len(stats) == 1 else axes
        for ax, (name, t) in zip(axes, ((n, v) for n, v in (("frc", frc_scores),
                                                             ("affinity", affinity),
                                                             ("triangles", triangles))
                                        if v is not None)):
            ax.hist(t.detach().float().flatten().cpu().numpy(), bins=100)
            ax.set_title(name)
        fig.savefig(save_path)
        plt.close(fig)
    return stats


def frc_flops(B: int, Hq: int, M: int, D: int) -> float:
    """Algorithmic FLOPs of compute_block_frc: 2 B Hq M^2 D + 2 B Hq M^3."""
    return 2.0 * B * Hq * M * M * D + 2.0 * B * Hq * math.pow(M, 3)
