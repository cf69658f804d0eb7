"""The prefill stages as registered PyTorch operators, ``torch.ops.cab.*``.

Each operator runs the same C-ABI entry point as the functional API
(``cab_attention.kernels``) and has a fake implementation that gives output shapes and
dtypes from the input metadata alone, so FakeTensor tracing and ``torch.compile`` can
place the operators in a graph without running them. The operators are registered for
CUDA tensors only: there is no CPU implementation.

    torch.ops.cab.coarsen_maxl2(q, k, block_size) -> (q_c, k_c, q_idx, k_idx)
    torch.ops.cab.block_frc(q_c, k_c, temperature, lambda_redundancy, formula,
                            normalization, redundancy_scale) -> frc
    torch.ops.cab.topk_blocks(frc, k, select_high, keep_diagonal, causal) -> (kv_idx, kv_num)
    torch.ops.cab.sparse_attn(q, k, v, kv_idx, kv_num, block_size, causal, softmax_scale) -> out
    torch.ops.cab.flash_attn(q, k, v, causal, softmax_scale, with_scores) -> (out, scores)

``softmax_scale <= 0`` means 1/sqrt(D). ``flash_attn`` returns the column scores of its
call (``[B, Hq, Nk]`` fp32, zeros when ``with_scores`` is false); accumulating them across
calls is left to the caller, as ``flash_attention_with_cumulative_scores`` does.
"""

from __future__ import annotations

import math
from typing import Tuple

import torch

from .kernels.coarsening import _coarsen
from .kernels.flash_attention_accumulate import flash_attention_forward
from .kernels.frc_kernel import compute_block_frc, topk_blocks
from .kernels.sparse_attention import block_sparse_attention

Tensor = torch.Tensor


def _scale(softmax_scale: float, D: int):
    return float(softmax_scale) if softmax_scale > 0 else 1.0 / math.sqrt(D)


@torch.library.custom_op("cab::coarsen_maxl2", mutates_args=(), device_types="cuda")
def coarsen_maxl2(q: Tensor, k: Tensor, block_size: int) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    qc, kc, qi, ki = _coarsen(q, k, int(block_size), True)
    return qc, kc, qi, ki


@coarsen_maxl2.register_fake
def _(q, k, block_size):
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    M = (N + block_size - 1) // block_size
    return (q.new_empty(B, Hq, M, D), k.new_empty(B, Hkv, M, D),
            q.new_empty(B, Hq, M, dtype=torch.int32), k.new_empty(B, Hkv, M, dtype=torch.int32))


@torch.library.custom_op("cab::block_frc", mutates_args=(), device_types="cuda")
def block_frc(q_c: Tensor, k_c: Tensor, temperature: float, lambda_redundancy: float, formula: str,
              normalization: str, redundancy_scale: str) -> Tensor:
    frc, _, _ = compute_block_frc(q_c, k_c, temperature, lambda_redundancy, formula, normalization,
                                  redundancy_scale, return_affinity=False, return_redundancy=False)
    return frc


@block_frc.register_fake
def _(q_c, k_c, temperature, lambda_redundancy, formula, normalization, redundancy_scale):
    B, Hq, M, _ = q_c.shape
    return q_c.new_empty(B, Hq, M, M, dtype=torch.float32)


@torch.library.custom_op("cab::topk_blocks", mutates_args=(), device_types="cuda")
def topk_blocks_op(frc: Tensor, k: int, select_high: bool, keep_diagonal: bool,
                   causal: bool) -> Tuple[Tensor, Tensor]:
    kv_idx, kv_num, _ = topk_blocks(frc, k, select_high, keep_diagonal, causal, return_dense=False)
    return kv_idx, kv_num


@topk_blocks_op.register_fake
def _(frc, k, select_high, keep_diagonal, causal):
    B, H, M, _ = frc.shape
    return frc.new_empty(B, H, M, k, dtype=torch.int32), frc.new_empty(B, H, M, dtype=torch.int32)


@torch.library.custom_op("cab::sparse_attn", mutates_args=(), device_types="cuda")
def sparse_attn(q: Tensor, k: Tensor, v: Tensor, kv_idx: Tensor, kv_num: Tensor, block_size: int,
                causal: bool, softmax_scale: float) -> Tensor:
    return block_sparse_attention(q, k, v, kv_idx, kv_num, int(block_size), causal,
                                  _scale(softmax_scale, q.shape[3]))


@sparse_attn.register_fake
def _(q, k, v, kv_idx, kv_num, block_size, causal, softmax_scale):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


@torch.library.custom_op("cab::flash_attn", mutates_args=(), device_types="cuda")
def flash_attn(q: Tensor, k: Tensor, v: Tensor, causal: bool, softmax_scale: float,
               with_scores: bool) -> Tuple[Tensor, Tensor]:
    B, Hq, _, D = q.shape
    scores = torch.zeros(B, Hq, k.shape[2], dtype=torch.float32, device=q.device)
    out = flash_attention_forward(q, k, v, scores=scores if with_scores else None,
                                  scale=_scale(softmax_scale, D), causal=causal)
    return out, scores


@flash_attn.register_fake
def _(q, k, v, causal, softmax_scale, with_scores):
    B, Hq, _, _ = q.shape
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            q.new_empty(B, Hq, k.shape[2], dtype=torch.float32))
