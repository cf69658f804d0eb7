"""torch.ops.cab.* on the GPU: each operator equals its functional-API call bit for bit
(the flash column scores up to float summation order),
passes torch.library.opcheck (schema, fake implementation, dispatch), and the chain
coarsen -> FRC -> top-k -> sparse attention traces into one graph under torch.compile
(fullgraph, AOT eager backend) with the eager result."""

import pytest
import torch

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import synthetic  # noqa: E402
from cab_attention.kernels import (block_sparse_attention, coarsen_qk_max_l2,  # noqa: E402
                                   compute_block_frc, flash_attention_forward, topk_blocks)


def _inputs():
    q, k, v = synthetic.make_qkv(1, 4, 2, 1000, 128, torch.bfloat16, seed=3)
    return q.cuda(), k.cuda(), v.cuda()


def test_ops_equal_functional_api():
    q, k, v = _inputs()
    qc, kc, qi, ki = torch.ops.cab.coarsen_maxl2(q, k, 64)
    qc2, kc2, qi2, ki2 = coarsen_qk_max_l2(q, k, 64, return_indices=True)
    assert torch.equal(qc, qc2) and torch.equal(kc, kc2) and torch.equal(qi, qi2) and torch.equal(ki, ki2)
    f = torch.ops.cab.block_frc(qc, kc, 1.0, 0.5, "additive", "abs", "none")
    f2, _, _ = compute_block_frc(qc, kc, 1.0, 0.5, "additive", "abs", "none")
    assert torch.equal(f, f2)
    idx, num = torch.ops.cab.topk_blocks(f, 3, True, True, False)
    idx2, num2, _ = topk_blocks(f, 3, True, True, False)
    assert torch.equal(idx, idx2) and torch.equal(num, num2)
    o = torch.ops.cab.sparse_attn(q, k, v, idx, num, 64, False, 0.0)
    assert torch.equal(o, block_sparse_attention(q, k, v, idx, num, 64))
    o3, s3 = torch.ops.cab.flash_attn(q, k, v, True, 0.0, True)
    s4 = torch.zeros_like(s3)
    o4 = flash_attention_forward(q, k, v, scores=s4, causal=True)
    assert torch.equal(o3, o4)
    # column scores are summed with float atomics across CTAs: equal up to summation order
    torch.testing.assert_close(s3, s4, rtol=1e-5, atol=1e-6)


def test_opcheck():
    q, k, v = _inputs()
    qc, kc, _, _ = torch.ops.cab.coarsen_maxl2(q, k, 64)
    f = torch.ops.cab.block_frc(qc, kc, 1.0, 0.5, "additive", "abs", "none")
    idx, num = torch.ops.cab.topk_blocks(f, 3, True, True, False)
    for op, args in ((torch.ops.cab.coarsen_maxl2.default, (q, k, 64)),
                     (torch.ops.cab.block_frc.default, (qc, kc, 1.0, 0.5, "additive", "abs", "none")),
                     (torch.ops.cab.topk_blocks.default, (f, 3, True, True, False)),
                     (torch.ops.cab.sparse_attn.default, (q, k, v, idx, num, 64, False, 0.0)),
                     (torch.ops.cab.flash_attn.default, (q, k, v, False, 0.0, True))):
        torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor"))


def test_compiled_chain_matches_eager():
    q, k, v = _inputs()

    def chain(q, k, v):
        qc, kc, _, _ = torch.ops.cab.coarsen_maxl2(q, k, 64)
        f = torch.ops.cab.block_frc(qc, kc, 1.0, 0.5, "additive", "abs", "none")
        idx, num = torch.ops.cab.topk_blocks(f, 3, True, True, False)
        return torch.ops.cab.sparse_attn(q, k, v, idx, num, 64, False, 0.0)

    eager = chain(q, k, v)
    compiled = torch.compile(chain, fullgraph=True, backend="aot_eager")(q, k, v)
    assert torch.equal(eager, compiled)
