"""Block-sparse attention against the reference's GPU path, FlexAttention (torch
``flex_attention``, compiled) fed the same kept-block lists through
``BlockMask.from_kv_blocks`` at BLOCK_SIZE 64 (oracle/flex_reference.py): an independent
second check of the kernel at the configs[1] shape (B2 H8 N32768 D128 bf16, s=0.95) and on
a causal grouped-query case (partial diagonal blocks). Max abs difference <= 2e-2."""

import pytest
import torch

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import CoarseCurvaturePredictor, _lib, synthetic  # noqa: E402
from cab_attention.kernels import block_sparse_attention  # noqa: E402
from oracle import flex_reference as fr  # noqa: E402


@pytest.mark.parametrize("B,Hq,Hkv,N,sp,causal", [
    (2, 8, 8, 32768, 0.95, False),   # configs[1]
    (1, 8, 2, 8192, 0.9, True),      # causal GQA
])
def test_matches_flex_attention(B, Hq, Hkv, N, sp, causal):
    q, k, v = (t.cuda() for t in synthetic.make_qkv(B, Hq, Hkv, N, 128, torch.bfloat16, 3))
    idx, num = CoarseCurvaturePredictor(64, sp, 0.5, causal=causal).predict_blocks(q, k)
    ours = block_sparse_attention(q, k, v, idx, num, 64, causal)
    flex = fr.attention(q, k, v, fr.block_mask(idx, num, N, 64, causal))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert (ours.float() - flex.float()).abs().max().item() <= 2e-2
