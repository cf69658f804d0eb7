"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Tolerances (from the path's stated bar): coarse indices and top-k index lists bit-exact;
FRC within 1e-2 relative (bf16/f16 inputs) or 1e-4 (fp32), relative to the largest
|F| of the (b, h) slice; attention max abs error <= 2e-2 (bf16/f16) or 1e-4 (fp32);
block-mask agreement >= 99.9% against the oracle's own FRC.
"""

import math

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import _lib  # noqa: E402
from cab_attention.kernels import (block_sparse_attention, coarsen_qk_max_l2,  # noqa: E402
                                   compute_block_frc, topk_blocks)
from cab_attention import synthetic  # noqa: E402

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert _lib.device_status() == 0, "a kernel's bounded wait timed out"


def rand(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def np_of(t):
    return t.detach().float().cpu().numpy()


# ------------------------------------------------------------------------- coarsening
@pytest.mark.parametrize("dt,B,Hq,Hkv,N,D,bs", [
    ("bf16", 2, 4, 4, 4096, 128, 64),
    ("bf16", 1, 8, 2, 1000, 64, 64),      # GQA, partial last block
    ("f16", 1, 2, 2, 777, 128, 32),
    ("f32", 1, 3, 3, 640, 64, 64),
    ("bf16", 1, 2, 1, 96, 256, 128),
    ("bf16", 1, 1, 1, 50, 64, 64),       # one partial block
])
def test_coarsen_bit_exact(dt, B, Hq, Hkv, N, D, bs):
    q = rand((B, Hq, N, D), DT[dt], 1)
    k = rand((B, Hkv, N, D), DT[dt], 2)
    # exact ties inside a block: duplicate a token, and a permuted copy (equal norm)
    q[0, 0, 1] = q[0, 0, 0]
    k[0, 0, 3] = k[0, 0, 2].flip(-1)
    # near tie: one element one ulp larger, so fp32 norms may tie but exact ones differ
    near = k[0, 0, 2].clone()
    near[0] = torch.nextafter(near[0].float(), torch.tensor(float("inf"))).to(near.dtype) \
        if DT[dt] == torch.float32 else (near[0].float() * (1 + 2 ** -7)).to(near.dtype)
    k[0, 0, 5] = near
    # a whole block of identical tokens: every fp32 norm ties, the lowest index wins
    if N >= 2 * bs:
        q[0, 0, bs:2 * bs] = q[0, 0, bs]
    qc, kc, qi, ki = coarsen_qk_max_l2(q.cuda(), k.cuda(), bs, return_indices=True)
    oq, oqi = orc.coarsen_maxl2(np_of(q), bs)
    ok, oki = orc.coarsen_maxl2(np_of(k), bs)
    assert np.array_equal(qi.cpu().numpy(), oqi)
    assert np.array_equal(ki.cpu().numpy(), oki)
    assert torch.equal(qc.cpu(), torch.from_numpy(oq).to(DT[dt]))
    assert torch.equal(kc.cpu(), torch.from_numpy(ok).to(DT[dt]))


def test_coarsen_strided_views():
    B, N, H, Dh = 2, 1024, 4, 64
    qkv = rand((B, N, 3 * H * Dh), torch.bfloat16, 5).cuda()
    t = qkv.view(B, N, 3, H, Dh)
    q, k = t[:, :, 0].transpose(1, 2), t[:, :, 1].transpose(1, 2)
    qc, kc, qi, ki = coarsen_qk_max_l2(q, k, 64, return_indices=True)
    _, oqi = orc.coarsen_maxl2(np_of(q), 64)
    _, oki = orc.coarsen_maxl2(np_of(k), 64)
    assert np.array_equal(qi.cpu().numpy(), oqi) and np.array_equal(ki.cpu().numpy(), oki)
    assert torch.equal(qc, q.contiguous().view(B, H, 16, 64, Dh)[
        torch.arange(B)[:, None, None], torch.arange(H)[None, :, None],
        torch.arange(16)[None, None, :], (qi % 64).long()])


# ------------------------------------------------------------------------- top-k
@pytest.mark.parametrize("M,k", [(1, 1), (7, 3), (64, 6), (130, 1), (512, 25), (333, 333), (2000, 100)])
@pytest.mark.parametrize("high,diag,causal", [(True, True, False), (False, False, False),
                                              (True, True, True), (False, True, True),
                                              (True, False, True)])
def test_topk_bit_exact(M, k, high, diag, causal):
    g = torch.Generator().manual_seed(M * 7 + k)
    F = torch.randint(-3, 4, (2, 2, M, M), generator=g).float()  # heavy ties
    F[0, 1] = torch.randn(M, M, generator=g)
    F[1, 0, :, ::3] = -0.0
    if M > 4:
        F[1, 1, 0, 2] = float("nan")
        F[1, 1, 1, :] = float("-inf")
    idx, num, dense = topk_blocks(F.cuda(), k, high, diag, causal)
    oidx, onum, odense = orc.topk_block_mask(F.numpy(), k, high, diag, causal)
    assert np.array_equal(num.cpu().numpy(), onum)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.array_equal(dense.cpu().numpy(), odense)


# ------------------------------------------------------------------------- FRC
@pytest.mark.parametrize("dt,B,Hq,Hkv,M,D", [
    ("bf16", 1, 2, 2, 64, 128),
    ("bf16", 2, 4, 2, 300, 64),
    ("f16", 1, 2, 1, 513, 128),
    ("bf16", 1, 1, 1, 1000, 128),
    ("f32", 1, 2, 2, 200, 64),
])
@pytest.mark.parametrize("norm,formula,rs", [("abs", "additive", "none"),
                                             ("minmax", "additive", "inv_m"),
                                             ("raw", "additive", "none"),
                                             ("abs", "multiplicative", "none")])
def test_frc_parity(dt, B, Hq, Hkv, M, D, norm, formula, rs):
    qc = rand((B, Hq, M, D), DT[dt], 11)
    kc = rand((B, Hkv, M, D), DT[dt], 12)
    f, a, r = compute_block_frc(qc.cuda(), kc.cuda(), 1.3, 0.5, formula, norm, rs)
    of, oa, orr = orc.block_frc(np_of(qc), np_of(kc), 1.3, 0.5, norm, formula, rs)
    tol = 1e-4 if dt == "f32" else 1e-2
    for got, want in ((f, of), (a, oa), (r, orr)):
        got = got.cpu().double().numpy()
        scale = np.abs(want).reshape(B * Hq, -1).max(axis=1).reshape(B, Hq, 1, 1) + 1e-30
        err = (np.abs(got - want) / scale).max()
        assert err <= tol, f"relative error {err:.3e} > {tol}"


def test_frc_mask_agreement_bf16():
    """Top-k on the GPU FRC vs top-k on the fp64 oracle FRC: >= 99.9% of blocks agree."""
    B, H, N, D = 1, 4, 2000 * 64 // 4, 128  # M = 500
    q, k, _ = synthetic.make_qkv(B, H, H, N, D, torch.bfloat16, seed=3)
    M = N // 64
    kk = orc.keep_count(M, 0.95)
    qc, kc = coarsen_qk_max_l2(q.cuda(), k.cuda(), 64)
    f, _, _ = compute_block_frc(qc, kc, return_affinity=False, return_redundancy=False)
    _, _, dense = topk_blocks(f, kk, True, True, False)
    of, _, _ = orc.block_frc(np_of(qc), np_of(kc), 1.0, 0.5, "abs")
    _, _, odense = orc.topk_block_mask(of, kk, True, True, False)
    d = dense.cpu().numpy()
    agree_all = (d == odense).mean()
    agree_kept = (d & odense).sum() / odense.sum()
    assert agree_all >= 0.999 and agree_kept >= 0.999, (agree_all, agree_kept)


# ------------------------------------------------------------------------- attention
def _lists(B, H, M, k, seed, causal, empty_rows=()):
    g = torch.Generator().manual_seed(seed)
    F = torch.randn(B, H, M, M, generator=g)
    idx, num, _ = orc.topk_block_mask(F.numpy(), k, True, True, causal)
    for (b, h, i) in empty_rows:
        num[b, h, i] = 0
        idx[b, h, i] = -1
    return idx, num


@pytest.mark.parametrize("dt,B,Hq,Hkv,N,D,bs,k,causal", [
    ("bf16", 1, 2, 2, 1024, 128, 64, 4, False),
    ("bf16", 1, 4, 2, 1000, 128, 64, 3, True),    # GQA, causal, partial block, odd M
    ("f16", 2, 2, 1, 704, 64, 64, 5, False),      # D=64
    ("bf16", 1, 1, 1, 8192, 128, 64, 16, False),  # many tiles per item
    ("bf16", 1, 2, 2, 130, 64, 64, 3, True),      # M=3
    ("f32", 1, 2, 2, 512, 64, 64, 3, True),       # CUDA-core path
    ("bf16", 1, 2, 2, 512, 64, 32, 5, False),     # block 32: CUDA-core path
])
def test_sparse_attention_parity(dt, B, Hq, Hkv, N, D, bs, k, causal):
    M = (N + bs - 1) // bs
    q = rand((B, Hq, N, D), DT[dt], 21)
    kk = rand((B, Hkv, N, D), DT[dt], 22)
    v = rand((B, Hkv, N, D), DT[dt], 23)
    idx, num = _lists(B, Hq, M, min(k, M), 24, causal, empty_rows=[(0, 0, M - 1)])
    out, lse = block_sparse_attention(q.cuda(), kk.cuda(), v.cuda(), torch.from_numpy(idx).cuda(),
                                      torch.from_numpy(num).cuda(), bs, causal, return_lse=True)
    want, wlse = orc.block_sparse_attention(np_of(q), np_of(kk), np_of(v), idx, num, bs, causal)
    tol = 1e-4 if dt == "f32" else 2e-2
    err = np.abs(out.cpu().double().numpy() - want).max()
    assert err <= tol, f"max abs err {err:.3e}"
    gl = lse.cpu().double().numpy()
    fin = np.isfinite(wlse)
    assert np.array_equal(np.isfinite(gl), fin)
    assert np.abs(gl[fin] - wlse[fin]).max() <= (1e-4 if dt == "f32" else 2e-2)
    # the row block with no kept key block is exactly zero
    r0 = (M - 1) * bs
    assert torch.all(out[0, 0, r0:] == 0)


def test_sparse_attention_into_strided_output():
    B, N, H, Dh = 1, 1024, 4, 64
    qkv = rand((B, N, 3 * H * Dh), torch.bfloat16, 31).cuda()
    t = qkv.view(B, N, 3, H, Dh)
    q, k, v = (t[:, :, i].transpose(1, 2) for i in range(3))
    M = N // 64
    idx, num = _lists(B, H, M, 4, 32, False)
    ctx = torch.empty(B, N, H * Dh, dtype=torch.bfloat16, device="cuda")
    block_sparse_attention(q, k, v, torch.from_numpy(idx).cuda(), torch.from_numpy(num).cuda(), 64,
                           out=ctx.view(B, N, H, Dh).transpose(1, 2))
    want, _ = orc.block_sparse_attention(np_of(q), np_of(k), np_of(v), idx, num, 64)
    got = ctx.view(B, N, H, Dh).transpose(1, 2).cpu().double().numpy()
    assert np.abs(got - want).max() <= 2e-2


# ------------------------------------------------------------------------- end to end
def test_predictor_c1_fp32_matches_oracle():
    """B1 H8 N4096 D64 fp32, s=0.90 -> identical masks and attention within 1e-4."""
    from cab_attention import CoarseCurvaturePredictor
    c = synthetic.make_config("c1", seed=0)
    pred = CoarseCurvaturePredictor(block_size=64, sparsity=c["sparsity"], lambda_redundancy=0.5)
    q, k, v = c["q"].cuda(), c["k"].cuda(), c["v"].cuda()
    mask, diag = pred(q, k, return_diagnostics=True)
    o = orc.predictor(np_of(c["q"]), np_of(c["k"]), 64, c["sparsity"], 0.5)
    assert (mask.cpu().numpy() == o["mask"]).mean() >= 0.999
    assert abs(diag["effective_sparsity"] - (1 - o["mask"].mean())) < 1e-3
    out = block_sparse_attention(q, k, v, diag["kv_indices"], diag["kv_num"], 64)
    want, _ = orc.block_sparse_attention(np_of(c["q"]), np_of(c["k"]), np_of(c["v"]),
                                         diag["kv_indices"].cpu().numpy(),
                                         diag["kv_num"].cpu().numpy(), 64)
    assert np.abs(out.cpu().double().numpy() - want).max() <= 1e-4


def test_planted_bridge_kept_c2_reduced():
    """configs[1] semantics at a quarter of N: the planted (i*, j*) is kept for every (b,h)."""
    from cab_attention import CoarseCurvaturePredictor
    c = synthetic.make_config("c2", seed=0)
    N = c["N"] // 4
    q, k = c["q"][:, :, :N].contiguous(), c["k"][:, :, :N].contiguous()
    M = N // 64
    g = torch.Generator().manual_seed(9)
    planted = []
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            (i, j), = synthetic.bridge_positions(M, 1, 1000 + b * 64 + h)
            synthetic.plant_bridge(q, k, b, h, i, j)
            planted.append((b, h, i, j))
    pred = CoarseCurvaturePredictor(block_size=64, sparsity=0.95, lambda_redundancy=0.5)
    mask = pred(q.cuda(), k.cuda()).cpu()
    for (b, h, i, j) in planted:
        assert mask[b, h, i, j], (b, h, i, j)


def test_cab_attention_layer_small():
    from cab_attention import CABAttention
    torch.manual_seed(0)
    layer = CABAttention(dim=256, num_heads=4, block_size=64, sparsity=0.9).cuda().to(torch.bfloat16)
    x = rand((2, 2048, 256), torch.bfloat16, 41).cuda()
    out, diag = layer(x, return_diagnostics=True)
    assert out.shape == x.shape and torch.isfinite(out).all()
    # oracle: same projections, oracle predictor, oracle attention
    qkv = layer.qkv(x)
    q, k, v = layer.split_heads(qkv)
    o = orc.predictor(np_of(q), np_of(k), 64, 0.9, 0.5)
    ctx, _ = orc.block_sparse_attention(np_of(q), np_of(k), np_of(v), o["kv_idx"], o["kv_num"], 64)
    agree = (diag["kv_indices"].cpu().numpy() == o["kv_idx"]).mean()
    assert agree >= 0.999
    if agree == 1.0:
        ctx_t = torch.from_numpy(ctx).float().transpose(1, 2).reshape(2, 2048, 256)
        want = ctx_t.to(torch.bfloat16).cuda() @ layer.proj.weight.t()
        assert (out.float() - want.float()).abs().max().item() <= 2e-2


# ------------------------------------------------------------------ hybrid (CAB V4) mask
@pytest.mark.parametrize("M,k,ratio", [(7, 3, 0.5), (64, 6, 0.25), (130, 13, 0.5), (333, 33, 1.0),
                                       (512, 25, 0.0), (2000, 100, 0.5), (257, 257, 0.3)])
@pytest.mark.parametrize("high,diag,causal", [(True, True, False), (False, False, False),
                                              (True, True, True), (True, False, True)])
def test_hybrid_topk_bit_exact(M, k, ratio, high, diag, causal):
    g = np.random.default_rng(M * 7 + k)
    scores = g.standard_normal((1, 2, M, M)).astype(np.float32)
    mag = g.random((1, 2, M, M)).astype(np.float32)
    # ties, NaN and signed zeros in both score matrices
    scores[0, 0, :, ::5] = scores[0, 0, :, :1]
    mag[0, 1, :, ::3] = 0.5
    scores[0, 1, 1, :4] = np.nan
    mag[0, 0, 2, :3] = np.nan
    scores[0, 1, 3, :6] = -0.0
    idx, num, dense = topk_blocks(torch.from_numpy(scores).cuda(), k, high, diag, causal,
                                  magnitude_scores=torch.from_numpy(mag).cuda(), magnitude_ratio=ratio)
    widx, wnum, wdense = orc.hybrid_block_mask(scores, mag, k, ratio, high, diag, causal)
    assert np.array_equal(num.cpu().numpy(), wnum)
    assert np.array_equal(idx.cpu().numpy(), widx)
    assert np.array_equal(dense.cpu().numpy(), wdense)


def test_generate_block_mask_hybrid_api():
    from cab_attention.kernels import generate_block_mask
    g = torch.Generator().manual_seed(3)
    frc = torch.randn(2, 4, 128, 128, generator=g)
    mag = torch.rand(2, 4, 128, 128, generator=g)
    dense, idx, num = generate_block_mask(frc.cuda(), sparsity=0.9, magnitude_scores=mag.cuda(),
                                          magnitude_ratio=0.5, return_indices=True)
    k = orc.keep_count(128, 0.9)
    widx, wnum, wdense = orc.hybrid_block_mask(frc.numpy(), mag.numpy(), k, 0.5)
    assert np.array_equal(dense.cpu().numpy(), wdense)
    assert np.array_equal(idx.cpu().numpy(), widx)


@pytest.mark.parametrize("dt,N,bs", [("f32", 256, 64), ("bf16", 300, 64), ("f16", 1000, 32),
                                     ("f32", 77, 8), ("bf16", 2048, 128)])
def test_block_max_pool_exact(dt, N, bs):
    from cab_attention.kernels import block_max_pool
    g = torch.Generator().manual_seed(N)
    attn = torch.softmax(torch.randn(1, 3, N, N, generator=g), dim=-1).to(DT[dt])
    attn[0, 1, :5, :7] = -1.0  # negative entries: a padded tile also sees its zero padding
    got = block_max_pool(attn.cuda(), bs)
    assert got.dtype == attn.dtype
    want = orc.block_max_pool(attn.float().numpy(), bs)
    assert np.array_equal(got.float().cpu().numpy(), want.astype(np.float32))
