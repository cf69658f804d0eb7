"""``CoarseCurvaturePredictor`` (``cab_attention/coarse_predictor.py`` of the reference).

API as used by ``README.md:117-128``, ``examples/demo_cab_attention.py:77-82,105-115,192-207``
and ``benchmarks/benchmark_predictor.py:59-63,114``:

    predictor = CoarseCurvaturePredictor(block_size=64, sparsity=0.95, lambda_redundancy=0.5)
    block_mask = predictor(q, k)                       # bool [B, H, M, M]
    block_mask, diag = predictor(q, k, return_diagnostics=True)
    predictor.estimate_flops(N, D)                     # {M, coarsening, matmul, triangles, total}

The pipeline is coarsen (K1) -> FRC (K2) -> per-row top-k (K3), all on sm_100a; each
stage is an NVTX range (``cab/coarsen``, ``cab/frc``, ``cab/topk``) for profilers.
``predict_blocks`` returns the index lists the sparse-attention kernel consumes without
materialising the dense mask or the diagnostics matrices. ``use_triton`` is accepted for
signature compatibility and ignored (there is one implementation).
"""

from __future__ import annotations

import torch
from torch import nn

from .kernels.coarsening import coarsen_qk_max_l2
from .kernels.frc_kernel import compute_block_frc, keep_count, topk_blocks


class CoarseCurvaturePredictor(nn.Module):
    def __init__(self, block_size: int = 64, sparsity: float = 0.95, lambda_redundancy: float = 0.5,
                 use_triton: bool = True, select_high: bool = True, keep_diagonal: bool = True,
                 causal: bool = False, normalization: str = "abs", formula: str = "additive",
                 temperature: float = 1.0, redundancy_scale: str = "none"):
        super().__init__()
        if not 0.0 <= sparsity < 1.0:
            raise ValueError("sparsity must be in [0, 1)")
        self.block_size = int(block_size)
        self.sparsity = float(sparsity)
        self.lambda_redundancy = float(lambda_redundancy)
        self.use_triton = use_triton  # accepted, ignored
        self.select_high = bool(select_high)
        self.keep_diagonal = bool(keep_diagonal)
        self.causal = bool(causal)
        self.normalization = normalization
        self.formula = formula
        self.temperature = float(temperature)
        self.redundancy_scale = redundancy_scale

    def num_blocks(self, seq_len: int) -> int:
        return (seq_len + self.block_size - 1) // self.block_size

    def keep_per_row(self, seq_len: int) -> int:
        return keep_count(self.num_blocks(seq_len), self.sparsity)

    def _scores(self, q, k, diagnostics: bool):
        with torch.cuda.nvtx.range("cab/coarsen"):
            qc, kc = coarsen_qk_max_l2(q, k, self.block_size)
        with torch.cuda.nvtx.range("cab/frc"):
            return compute_block_frc(qc, kc, self.temperature, self.lambda_redundancy, self.formula,
                                     self.normalization, self.redundancy_scale,
                                     return_affinity=diagnostics, return_redundancy=diagnostics)

    @torch.no_grad()
    def predict_blocks(self, q: torch.Tensor, k: torch.Tensor, return_dense: bool = False):
        """``(kv_idx [B,Hq,M,k] int32, kv_num [B,Hq,M] int32[, dense bool])``."""
        frc, _, _ = self._scores(q, k, diagnostics=False)
        with torch.cuda.nvtx.range("cab/topk"):
            kv_idx, kv_num, dense = topk_blocks(frc, self.keep_per_row(q.shape[2]), self.select_high,
                                                self.keep_diagonal, self.causal,
                                                return_dense=return_dense)
        return (kv_idx, kv_num, dense) if return_dense else (kv_idx, kv_num)

    @torch.no_grad()
    def forward(self, q: torch.Tensor, k: torch.Tensor, return_diagnostics: bool = False):
        frc, aff, red = self._scores(q, k, diagnostics=return_diagnostics)
        with torch.cuda.nvtx.range("cab/topk"):
            kv_idx, kv_num, dense = topk_blocks(frc, self.keep_per_row(q.shape[2]), self.select_high,
                                                self.keep_diagonal, self.causal, return_dense=True)
        if not return_diagnostics:
            return dense
        diag = {
            "effective_sparsity": 1.0 - dense.float().mean().item(),
            "num_blocks": dense.shape[-1],
            "blocks_per_row": int(kv_idx.shape[-1]),
            "frc_scores": frc,
            "affinity": aff,
            "triangles": red,
            "kv_indices": kv_idx,
            "kv_num": kv_num,
        }
        return dense, diag

    def estimate_flops(self, N: int, D: int) -> dict:
        """Per-(b, h) FLOP counts: coarsening 4ND (norms of Q and K), affinity 2M^2 D,
        triangles 2M^3."""
        M = self.num_blocks(N)
        coarse = 4 * N * D
        matmul = 2 * M * M * D
        tri = 2 * M ** 3
        return {"M": M, "coarsening": coarse, "matmul": matmul, "triangles": tri,
                "total": coarse + matmul + tri}

    def extra_repr(self) -> str:
        return (f"block_size={self.block_size}, sparsity={self.sparsity}, "
                f"lambda_redundancy={self.lambda_redundancy}, select_high={self.select_high}, "
                f"keep_diagonal={self.keep_diagonal}, causal={self.causal}, "
                f"normalization={self.normalization!r}, formula={self.formula!r}")
