"""Three-component eviction policy (``cab_attention/eviction/policy.py`` of the reference)
on the sm_100a kernel ``cab_evict_select``.

Keeps the local window, the highest-importance tokens and "bridge" tokens (moderate
importance, or strongest two-way connectivity with the important tokens when an attention
matrix is given) and returns the kept positions sorted, as ``select_indices`` does
(``policy.py:40-210``). The whole selection is one to four kernel launches with no host
synchronisation; ``select_indices`` itself reads back four counters to return the exact-length
index tensor and the diagnostics, like the reference. Ties go to the lower position
(``torch.topk`` leaves their order unspecified).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from .. import _lib


@dataclass
class EvictionConfig:
    """Budget shares of the three components (must sum to 1)."""
    local_ratio: float = 0.3
    bridge_ratio: float = 0.2
    importance_ratio: float = 0.5

    def __post_init__(self):
        total = self.local_ratio + self.bridge_ratio + self.importance_ratio
        assert abs(total - 1.0) < 1e-6, f"Ratios must sum to 1.0, got {total}"


def select_indices_batched(cache_len: int, keep_size: int, importance: Optional[torch.Tensor],
                           attention: Optional[torch.Tensor] = None, local_ratio: float = 0.3,
                           bridge_ratio: float = 0.2, device=None, batch: Optional[int] = None):
    """Batched selection without host synchronisation: ``importance [batch, n]`` (or None),
    ``attention [batch, L, L]`` (or None) -> ``(keep [batch, keep_size] int64 ascending,
    -1 padded; counts [batch, 4] int32 = kept, local, importance, bridge)``. ``batch`` is
    needed only when neither tensor is given (positional selection)."""
    ref = importance if importance is not None else attention
    dev = ref.device if ref is not None else torch.device(
        "cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _lib.require_cuda(torch.empty(0, device=dev))
    if batch is None:
        batch = ref.shape[0] if ref is not None else 1
    imp = imp_len = None
    if importance is not None:
        imp = importance.float().contiguous()
        imp_len = imp.shape[-1]
        if imp.dim() != 2 or imp.shape[0] != batch:
            raise ValueError("importance must be [batch, n]")
    att = None
    if attention is not None:
        att = attention.float().contiguous()
        if tuple(att.shape) != (batch, cache_len, cache_len):
            raise ValueError(f"attention must be [batch, {cache_len}, {cache_len}]")
    keep = torch.empty(batch, keep_size, dtype=torch.int64, device=dev)
    counts = torch.empty(batch, 4, dtype=torch.int32, device=dev)
    L = _lib.lib()
    nbytes = _lib._c_size(0)
    _lib.check(L.cab_evict_workspace_size(batch, cache_len, int(att is not None), nbytes),
               "cab_evict_workspace_size")
    ws = _lib.workspace(nbytes.value, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = L.cab_evict_select(_lib.ptr(imp), imp_len or 0, _lib.ptr(att), batch, cache_len, keep_size,
                            float(local_ratio), float(bridge_ratio), keep.data_ptr(), counts.data_ptr(),
                            _lib.ptr(ws), nbytes.value, stream)
    _lib.check(rc, "cab_evict_select")
    return keep, counts


class ThreeComponentEvictionPolicy:
    """Local window + importance (H2O-style cumulative attention) + bridges."""

    def __init__(self, config: EvictionConfig):
        self.config = config

    def select_indices(self, cache_len: int, keep_size: int, importance_scores: Optional[torch.Tensor],
                       attention_matrix: Optional[torch.Tensor] = None, device: str = "cuda"
                       ) -> Tuple[torch.Tensor, dict]:
        """``(keep_indices [n] int64 sorted, diagnostics)`` for one sequence."""
        imp = importance_scores.reshape(1, -1) if importance_scores is not None else None
        att = attention_matrix.reshape(1, cache_len, cache_len) if attention_matrix is not None else None
        keep, counts = select_indices_batched(cache_len, keep_size, imp, att, self.config.local_ratio,
                                              self.config.bridge_ratio, device=device)
        n, n_local, n_imp, n_bridge = (int(x) for x in counts[0].tolist())
        keep = keep[0, :n]
        frac = (lambda c: c / n) if n > 0 else (lambda c: 0)
        diagnostics = {
            "cache_len": cache_len,
            "keep_size": n,
            "local_count": n_local,
            "importance_count": n_imp,
            "bridge_count": n_bridge,
            "local_ratio_actual": frac(n_local),
            "importance_ratio_actual": frac(n_imp),
            "bridge_ratio_actual": frac(n_bridge),
        }
        return keep, diagnostics
