"""``CABAttention`` (``cab_attention/cab_attention.py`` of the reference).

API as used by ``README.md:77-111`` and ``examples/demo_cab_attention.py:37-63``:

    attn = CABAttention(dim=512, num_heads=8, block_size=64, sparsity=0.95)
    out = attn(x)                                   # x [B, N, dim] -> [B, N, dim]
    out, diag = attn(x, return_diagnostics=True)    # effective_sparsity, num_blocks,
                                                    # frc_scores, affinity, triangles

Layer: fused QKV projection -> CoarseCurvaturePredictor (K1-K3) -> block-sparse attention
(K4) -> output projection. Q, K and V are strided head views of the fused projection
output and the attention writes straight into the [B, N, dim] layout the output
projection reads, so no transpose is materialised. The projections are plain dense
GEMMs (torch / cuBLAS); weights are initialised N(0, 0.02^2) without bias.
"""

from __future__ import annotations

import torch
from torch import nn

from .coarse_predictor import CoarseCurvaturePredictor
from .kernels.sparse_attention import block_sparse_attention


class CABAttention(nn.Module):
    def __init__(self, dim: int, num_heads: int, block_size: int = 64, sparsity: float = 0.95,
                 lambda_redundancy: float = 0.5, causal: bool = False, select_high: bool = True,
                 keep_diagonal: bool = True, qkv_bias: bool = False, init_std: float = 0.02,
                 **predictor_kwargs):
        super().__init__()
        if dim % num_heads:
            raise ValueError("dim must be divisible by num_heads")
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.block_size = block_size
        self.causal = causal
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim, bias=qkv_bias)
        self.predictor = CoarseCurvaturePredictor(block_size=block_size, sparsity=sparsity,
                                                  lambda_redundancy=lambda_redundancy,
                                                  select_high=select_high,
                                                  keep_diagonal=keep_diagonal, causal=causal,
                                                  **predictor_kwargs)
        self.init_std = init_std
        self.reset_parameters()

    def reset_parameters(self, generator: torch.Generator | None = None) -> None:
        with torch.no_grad():
            for lin in (self.qkv, self.proj):
                lin.weight.normal_(0.0, self.init_std, generator=generator)
                if lin.bias is not None:
                    lin.bias.zero_()

    def split_heads(self, qkv: torch.Tensor):
        """[B, N, 3*dim] -> three strided [B, H, N, Dh] views."""
        B, N, _ = qkv.shape
        t = qkv.view(B, N, 3, self.num_heads, self.head_dim)
        return (t[:, :, 0].transpose(1, 2), t[:, :, 1].transpose(1, 2),
                t[:, :, 2].transpose(1, 2))

    def forward(self, x: torch.Tensor, return_diagnostics: bool = False):
        B, N, dim = x.shape
        with torch.cuda.nvtx.range("cab/qkv_proj"):
            qkv = self.qkv(x)
        q, k, v = self.split_heads(qkv)
        if return_diagnostics:
            dense, diag = self.predictor(q, k, return_diagnostics=True)
            kv_idx, kv_num = diag["kv_indices"], diag["kv_num"]
        else:
            kv_idx, kv_num = self.predictor.predict_blocks(q, k)
        ctx = torch.empty(B, N, dim, dtype=x.dtype, device=x.device)
        ctx_heads = ctx.view(B, N, self.num_heads, self.head_dim).transpose(1, 2)
        with torch.cuda.nvtx.range("cab/sparse_attention"):
            block_sparse_attention(q, k, v, kv_idx, kv_num, self.block_size, causal=self.causal,
                                   out=ctx_heads)
        with torch.cuda.nvtx.range("cab/out_proj"):
            out = self.proj(ctx)
        if return_diagnostics:
            return out, diag
        return out
