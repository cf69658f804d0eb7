"""Algorithmic work of each stage of the path and its roofline fraction.

Bytes (HBM-bound stages) and FLOPs (tensor-bound stages) are the algorithmic amounts:
each input read once, each output written once, useful multiply-adds only.

- coarsening (HBM): read (B*Hq + B*Hkv) * N * D * s, write (B*Hq + B*Hkv) * M * (D * s [+ 4])
- coarse FRC (tensor): 2 * B * Hq * M^2 * D (affinity) + 2 * B * Hq * M^3 (triangles)
- top-k (HBM): B * H * M^2 * 4 read + B * H * M * (k + 1) * 4 written
- block-sparse attention (tensor): 4 * bs^2 * D per kept (query block, key block) pair
- dense flash attention (tensor): 4 * B * Hq * Nq * Nk * D
- node FRC (HBM): batch * N^2 * s read once
"""

from __future__ import annotations

import json
from pathlib import Path

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def coarsen_bytes(B, Hq, Hkv, N, D, elem_size=2, block_size=64, with_indices=False):
    M = (N + block_size - 1) // block_size
    per_row = D * elem_size + (4 if with_indices else 0)
    return (B * Hq + B * Hkv) * (N * D * elem_size + M * per_row)


def frc_flops(B, Hq, M, D):
    return 2.0 * B * Hq * M * M * D + 2.0 * B * Hq * M ** 3


def topk_bytes(B, H, M, k):
    return B * H * M * M * 4 + B * H * M * (k + 1) * 4


def sparse_attention_flops(kept_block_pairs, block_size, D):
    return 4.0 * block_size * block_size * D * kept_block_pairs


def flash_attention_flops(B, Hq, Nq, Nk, D):
    return 4.0 * B * Hq * Nq * Nk * D


def node_frc_bytes(batch, N, elem_size=4):
    return batch * N * N * elem_size


def measured_peaks(path=None):
    """``(peaks dict, "measured" | "fallback")`` from MEASURED_PEAKS.json next to the repo."""
    p = Path(path) if path else Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d.setdefault("bf16_tflops_sustained", d.get("bf16_tflops"))
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def fraction(work, ms, peak, unit):
    """Achieved rate of `work` (bytes or FLOPs) in `ms` and its fraction of `peak`
    (`unit` "GB/s" or "TFLOP/s")."""
    scale = 1e6 if unit == "GB/s" else 1e9
    achieved = work / ms / scale
    return achieved, achieved / peak
