"""Full-size configurations through the public API: the north_star layer itself (B2 H8
N128000 D128 bf16, s=0.95, k=100; the workload bench.py times, through the bench step's own
calls), configs[1] (C2: B2 H8 N32768 D128 bf16,
s=0.95, one planted bridge per (b, h)), configs[2] (C3: the CABAttention layer, dim 512,
8 heads of 64, B2 N128000 bf16, s=0.95, projection weights N(0, 0.02^2)), configs[3] (C4:
the predictor over N in {1k, 4k, 16k, 64k, 128k}, B2 H8 D128 bf16, s=0.95) and configs[4]
(C5: GQA 32/8, B1 N65536 D128 bf16, causal, s=0.99, four planted bridges). Checked by
size-independent properties: every planted bridge is kept; on sampled heads the block
mask agrees with the float64 oracle on >= 99.9 % of all blocks and of kept blocks (fp16
triangle products move a few near-tied blocks: 99.94-100 % of kept blocks measured on every
configuration); attention on sampled query blocks
matches the oracle given the same lists (max abs error <= 2e-2); the layer output on
sampled rows matches the output projection of the oracle attention (max abs error
<= 2e-3 at these weight scales)."""

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import CABAttention, CoarseCurvaturePredictor, _lib, synthetic  # noqa: E402
from cab_attention.kernels import block_sparse_attention  # noqa: E402


@pytest.mark.parametrize("name", ["c2", "c5"])
def test_full_size_config(name):
    c = synthetic.make_config(name, seed=0)
    q_h, k_h, v_h = c["q"], c["k"], c["v"]
    q, k, v = q_h.cuda(), k_h.cuda(), v_h.cuda()
    pred = CoarseCurvaturePredictor(64, c["sparsity"], 0.5, causal=c["causal"])
    kv_idx, kv_num, dense = pred.predict_blocks(q, k, return_dense=True)
    out = block_sparse_attention(q, k, v, kv_idx, kv_num, 64, causal=c["causal"])
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    d = dense.cpu().numpy()
    assert c["bridges_planted"]
    for (b, h, i, j) in c["bridges_planted"]:
        assert d[b, h, i, j], (b, h, i, j)
    G = c["Hq"] // c["Hkv"]
    heads = [(0, 0), (c["B"] - 1, c["Hq"] - 1)] + [(b, h) for (b, h, _, _) in c["bridges_planted"][:1]]
    idx_h, num_h = kv_idx.cpu().numpy(), kv_num.cpu().numpy()
    for (b, h) in heads:
        qs = q_h[b:b + 1, h:h + 1].float().numpy()
        ks = k_h[b:b + 1, h // G:h // G + 1].float().numpy()
        vs = v_h[b:b + 1, h // G:h // G + 1].float().numpy()
        o = orc.predictor(qs, ks, 64, c["sparsity"], 0.5, causal=c["causal"])
        want = o["mask"][0, 0]
        got = d[b, h]
        assert (got == want).mean() >= 0.999
        assert (got & want).sum() / want.sum() >= 0.999
        M = c["M"]
        rows = [(0, 0, i) for i in (0, 1, M // 3, M // 2 + 1, M - 2, M - 1)]
        att, _ = orc.block_sparse_attention(qs, ks, vs, idx_h[b:b + 1, h:h + 1], num_h[b:b + 1, h:h + 1], 64,
                                            c["causal"], rows=rows)
        got_o = out[b, h].float().cpu().numpy()
        for (_, _, i) in rows:
            r0, r1 = 64 * i, min(c["N"], 64 * (i + 1))
            err = np.abs(got_o[r0:r1] - att[0, 0, r0:r1]).max()
            assert err <= 2e-2, (b, h, i, err)


def _lists_to_dense(idx, num, M):
    got = np.zeros((M, M), dtype=bool)
    for i in range(M):
        got[i, idx[i, :num[i]]] = True
    return got


def test_north_star_layer():
    """The benchmarked workload, with the exact stage calls of bench.Layer.stages: coarsen
    -> FRC -> top-k (k = 100 of M = 2000) -> block-sparse attention. On two sampled heads
    the block mask agrees with the float64 oracle on >= 99.9 % of all blocks and of kept
    blocks, and attention on six sampled query blocks per head matches the oracle given the
    same lists (max abs error <= 2e-2)."""
    import bench
    cfg = bench.CONFIGS["ns"]
    q_h, k_h, v_h = bench.make_inputs(cfg, 0, 0, pin=False)
    q, k, v = q_h.cuda(), k_h.cuda(), v_h.cuda()
    out, kv_idx, kv_num = bench.Layer(cfg).stages(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    B, H, N = cfg["B"], cfg["Hq"], cfg["N"]
    M = (N + 63) // 64
    kk = orc.keep_count(M, cfg["sparsity"])
    assert kk == 100 and tuple(kv_idx.shape) == (B, H, M, kk) and bool((kv_num == kk).all())
    idx_h, num_h = kv_idx.cpu().numpy(), kv_num.cpu().numpy()
    assert (np.diff(idx_h, axis=-1) > 0).all()  # ascending, no duplicates
    rows = [(0, 0, i) for i in (0, 1, M // 3, M // 2 + 1, M - 2, M - 1)]
    for (b, h) in [(0, 0), (B - 1, H - 1)]:
        qs = q_h[b:b + 1, h:h + 1].float().numpy()
        ks = k_h[b:b + 1, h:h + 1].float().numpy()
        vs = v_h[b:b + 1, h:h + 1].float().numpy()
        want = orc.predictor(qs, ks, 64, cfg["sparsity"], 0.5)["mask"][0, 0]
        got = _lists_to_dense(idx_h[b, h], num_h[b, h], M)
        assert (got == want).mean() >= 0.999
        assert (got & want).sum() / want.sum() >= 0.999
        att, _ = orc.block_sparse_attention(qs, ks, vs, idx_h[b:b + 1, h:h + 1], num_h[b:b + 1, h:h + 1], 64,
                                            False, rows=rows)
        got_o = out[b, h].float().cpu().numpy()
        for (_, _, i) in rows:
            err = np.abs(got_o[64 * i:64 * (i + 1)] - att[0, 0, 64 * i:64 * (i + 1)]).max()
            assert err <= 2e-2, (b, h, i, err)


def _mask_agrees(got, want, kept_bar=0.999):
    assert (got == want).mean() >= 0.999
    assert (got & want).sum() / max(1, want.sum()) >= kept_bar


def test_c3_cab_attention_layer():
    B, N, dim, H = 2, 128000, 512, 8
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, N, dim, generator=g).to(torch.bfloat16)
    layer = CABAttention(dim, H, block_size=64, sparsity=0.95, lambda_redundancy=0.5)
    layer.reset_parameters(torch.Generator().manual_seed(1))
    layer = layer.to(torch.bfloat16).cuda()
    xd = x.cuda()
    with torch.no_grad():
        out, diag = layer(xd, return_diagnostics=True)
        q, k, v = layer.split_heads(layer.qkv(xd))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert out.shape == (B, N, dim) and torch.isfinite(out).all()
    M = (N + 63) // 64
    assert diag["num_blocks"] == M and diag["blocks_per_row"] == orc.keep_count(M, 0.95)
    idx_h, num_h = diag["kv_indices"].cpu().numpy(), diag["kv_num"].cpu().numpy()
    assert tuple(diag["kv_num"].shape) == (B, H, M)
    out_h = out.float().cpu().numpy()
    w_o = layer.proj.weight.detach().float().cpu().numpy()
    for (b, h) in [(0, 0), (1, H - 1)]:
        qs = q[b:b + 1, h:h + 1].float().cpu().numpy()
        ks = k[b:b + 1, h:h + 1].float().cpu().numpy()
        o = orc.predictor(qs, ks, 64, 0.95, 0.5)
        got = np.zeros((M, M), dtype=bool)
        for i in range(M):
            got[i, idx_h[b, h, i, :num_h[b, h, i]]] = True
        _mask_agrees(got, o["mask"][0, 0])
    # attention of every head on sampled query blocks (the layer's own lists), then the
    # output projection of the oracle context against the layer output on those rows
    rows = [(0, 0, i) for i in (0, 1, M // 2, M - 1)]
    for b in range(B):
        ctx = np.zeros((len(rows), 64, dim), dtype=np.float64)
        for h in range(H):
            qs = q[b:b + 1, h:h + 1].float().cpu().numpy()
            ks = k[b:b + 1, h:h + 1].float().cpu().numpy()
            vs = v[b:b + 1, h:h + 1].float().cpu().numpy()
            att, _ = orc.block_sparse_attention(qs, ks, vs, idx_h[b:b + 1, h:h + 1], num_h[b:b + 1, h:h + 1],
                                                64, False, rows=rows)
            for n, (_, _, i) in enumerate(rows):
                ctx[n, :, 64 * h:64 * (h + 1)] = att[0, 0, 64 * i:64 * (i + 1)]
        for n, (_, _, i) in enumerate(rows):
            want = ctx[n] @ w_o.T.astype(np.float64)
            err = np.abs(out_h[b, 64 * i:64 * (i + 1)] - want).max()
            assert err <= 2e-3, (b, i, err)


@pytest.mark.parametrize("N", [1024, 4096, 16384, 65536, 131072])
def test_c4_predictor_sweep(N):
    q, k, _ = synthetic.make_qkv(2, 8, 8, N, 128, torch.bfloat16, 0)
    pred = CoarseCurvaturePredictor(64, 0.95, 0.5)
    kv_idx, kv_num, dense = pred.predict_blocks(q.cuda(), k.cuda(), return_dense=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    M = (N + 63) // 64
    kk = orc.keep_count(M, 0.95)
    assert kv_idx.shape == (2, 8, M, kk) and bool((kv_num == kk).all())
    d = dense.cpu().numpy()
    for (b, h) in [(0, 0), (1, 7)]:
        o = orc.predictor(q[b:b + 1, h:h + 1].float().numpy(), k[b:b + 1, h:h + 1].float().numpy(),
                          64, 0.95, 0.5)
        _mask_agrees(d[b, h], o["mask"][0, 0])
