"""The CPU oracle against fixtures produced by the reference's own code (CPU only)."""

import numpy as np
import pytest

from oracle import cab_oracle as orc


def test_edge_frc_matches_test_ipynb(golden_dir):
    g = np.load(golden_dir / "test_ipynb_bridge.npz")
    frc = orc.edge_frc_augmented(g["adj"])
    np.testing.assert_allclose(frc, g["frc"], rtol=1e-5, atol=1e-3)
    u, v = g["bridge"]
    assert round(float(frc[u, v]), 2) == -85.71  # test.ipynb published output


def test_notebook_keep_pattern(golden_dir):
    g = np.load(golden_dir / "test_ipynb_bridge.npz")
    frc = orc.edge_frc_augmented(g["adj"])
    u, v = g["bridge"]
    for s, h2o, cab in zip(g["sparsities"], g["h2o_masks"], g["cab_masks"]):
        mh = orc.notebook_topk_mask(g["adj"], s, largest=True)
        mc = orc.notebook_topk_mask(frc, s, largest=False)
        assert (mh == h2o).all()
        assert (mc == cab).all()
        assert mc[u, v]  # CAB keeps the bridge at every sparsity (test.ipynb output)
    # H2O loses the bridge from 80% up (test.ipynb output)
    assert [bool(m[u, v]) for m in g["h2o_masks"]] == [True] + [False] * 5


def test_colab_v3_pipeline(golden_dir):
    g = np.load(golden_dir / "colab_v3_pipeline.npz")
    for c in range(2):
        q, k, v = g[f"c{c}_q"], g[f"c{c}_k"], g[f"c{c}_v"]
        bs, kept = int(g[f"c{c}_meta"][0]), int(g[f"c{c}_meta"][1])
        sp = float(g[f"c{c}_sparsity"])
        qc, _ = orc.coarsen_maxl2(q, bs)
        kc, _ = orc.coarsen_maxl2(k, bs)
        frc, _, _ = orc.block_frc(qc, kc, lambda_redundancy=0.5, normalization="abs")
        mask = orc.global_threshold_mask(frc, sp)
        assert int(mask.sum()) == kept
        out = orc.dense_masked_attention(q, k, v, mask, bs)
        np.testing.assert_allclose(out, g[f"c{c}_out"], rtol=1e-4, atol=1e-5)
        # the block-list attention gives the same numbers as the dense expansion
        kv_idx, kv_num = orc.dense_to_lists(mask)
        out2, _ = orc.block_sparse_attention(q, k, v, kv_idx, kv_num, bs)
        np.testing.assert_allclose(out2, out, rtol=1e-9, atol=1e-10)


def test_methods_cabv3_masked_softmax(golden_dir):
    g = np.load(golden_dir / "methods_cabv3.npz")
    bs, sp, lam = int(g["params"][0]), float(g["params"][1]), float(g["params"][2])
    q, k = g["q"], g["k"]
    qc, _ = orc.coarsen_maxl2(q, bs)
    kc, _ = orc.coarsen_maxl2(k, bs)
    frc, _, _ = orc.block_frc(qc, kc, lambda_redundancy=lam, normalization="abs")
    M = frc.shape[-1]
    _, _, dense = orc.topk_block_mask(frc, orc.keep_count(M, sp), True, True, True)
    tok = orc.expand_block_mask(dense, bs, q.shape[2])
    s = np.where(tok, g["logits"].astype(np.float64), -np.inf)
    m = s.max(-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        w = np.exp(s - m)
        w = w / w.sum(-1, keepdims=True)
    w = np.nan_to_num(w, nan=0.0)
    np.testing.assert_allclose(w, g["weights"], rtol=1e-5, atol=1e-6)
    # the same numbers through the block-list attention path (V = identity picks weights)
    N = q.shape[2]
    kv_idx, kv_num, _ = orc.topk_block_mask(frc, orc.keep_count(M, sp), True, True, True)
    eye = np.broadcast_to(np.eye(N), (1, 2, N, N)).copy()
    out, _ = orc.block_sparse_attention(q, k, eye, kv_idx, kv_num, bs, causal=True)
    np.testing.assert_allclose(out, g["weights"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("keep_diag,causal", [(False, False), (True, False), (True, True),
                                              (False, True)])
def test_topk_semantics_small(keep_diag, causal):
    rng = np.random.default_rng(3)
    F = rng.integers(0, 4, size=(1, 1, 9, 9)).astype(np.float32)  # many ties
    k = 3
    for high in (True, False):
        idx, num, dense = orc.topk_block_mask(F, k, high, keep_diag, causal)
        for i in range(9):
            cand = list(range(i + 1)) if causal else list(range(9))
            key = [(F[0, 0, i, j] if high else -F[0, 0, i, j]) for j in cand]
            order = sorted(cand, key=lambda j: (-(1 if (keep_diag and j == i) else 0),
                                                -key[cand.index(j)], j))
            want = sorted(order[:min(k, len(cand))])
            assert list(idx[0, 0, i, : num[0, 0, i]]) == want
            assert dense[0, 0, i].sum() == len(want)


def test_keep_count_matches_configs():
    assert orc.keep_count(64, 0.90) == 6
    assert orc.keep_count(512, 0.95) == 25
    assert orc.keep_count(2000, 0.95) == 100
    assert orc.keep_count(1024, 0.99) == 10
    assert orc.keep_count(16, 0.999) == 1


def test_coarsen_tie_and_partial_block():
    x = np.zeros((1, 1, 10, 4), dtype=np.float32)
    x[0, 0, 1] = [1, 0, 0, 0]
    x[0, 0, 2] = [0, 1, 0, 0]   # tie with token 1 -> token 1 wins
    x[0, 0, 9] = [0, 0, 2, 0]   # partial last block (tokens 8, 9)
    xc, idx = orc.coarsen_maxl2(x, 4)
    assert idx.tolist() == [[[1, 4, 9]]]
    assert (xc[0, 0, 2] == x[0, 0, 9]).all()


def test_flash_cumulative_matches_reference_kernel(golden_dir):
    """The flash restatement against the reference Triton kernel's own outputs
    (tests/golden/make_flash_golden.py): output to the fp16/bf16 P.V rounding the kernel
    applies, cumulative column scores to 1e-4 of the largest score."""
    import torch

    g = np.load(golden_dir / "flash_cumulative.npz")
    for name in g["names"]:
        dtype = {"float16": torch.float16, "bfloat16": torch.bfloat16}[str(g[f"{name}/dtype"])]
        q, k, v = (g[f"{name}/{x}"] for x in "qkv")
        init = g[f"{name}/init"]
        start = None
        if init.shape[2]:
            start = np.zeros(g[f"{name}/cum"].shape)
            start[:, :, : init.shape[2]] = init
        out, cum = orc.flash_attention_cumulative(
            q, k, v, scores=start, p_round=lambda p: torch.from_numpy(p).to(dtype).double().numpy())
        tol = 5e-3 if dtype == torch.float16 else 2e-2
        assert np.abs(out - g[f"{name}/out"]).max() <= tol, name
        ref = g[f"{name}/cum"].astype(np.float64)
        assert np.abs(cum - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max()), name


def test_hybrid_limits_reduce_to_plain_topk():
    """ratio 0 selects by FRC only, ratio 1 by magnitude only (diagonal still forced)."""
    g = np.random.default_rng(11)
    f = g.standard_normal((1, 1, 50, 50)).astype(np.float32)
    m = g.standard_normal((1, 1, 50, 50)).astype(np.float32)
    for causal in (False, True):
        i0, n0, d0 = orc.hybrid_block_mask(f, m, 7, 0.0, True, True, causal)
        j0, _, _ = orc.topk_block_mask(f, 7, True, True, causal)
        assert np.array_equal(i0, j0)
        i1, n1, d1 = orc.hybrid_block_mask(f, m, 7, 1.0, True, True, causal)
        j1, _, _ = orc.topk_block_mask(m, 7, True, True, causal)
        assert np.array_equal(i1, j1)
        i5, n5, d5 = orc.hybrid_block_mask(f, m, 7, 0.5, True, True, causal)
        assert (d5.sum(-1) == n5).all() and all(d5[0, 0, i, i] for i in range(50))


def test_node_frc_matches_reference(golden_dir):
    """Node-level FRC restatement against the reference's compute_frc_pytorch outputs."""
    g = np.load(golden_dir / "node_frc.npz")
    for name in g["names"]:
        frc, _, _ = orc.node_frc(g[f"{name}/attention"])
        ref = g[f"{name}/frc"].astype(np.float64)
        assert np.abs(frc - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), name


def test_evict_select_matches_reference(golden_dir):
    """The eviction restatement against the reference's select_indices outputs."""
    g = np.load(golden_dir / "evict_select.npz")
    for name in g["names"]:
        L, K, lr, br = g[f"{name}/params"]
        imp = g[f"{name}/importance"]
        att = g[f"{name}/attention"]
        keep, counts = orc.evict_select(int(L), int(K), imp if imp.size else None, att if att.size else None,
                                        lr, br)
        assert np.array_equal(keep, g[f"{name}/keep"]), name
        assert tuple(counts) == tuple(int(x) for x in g[f"{name}/counts"]), name
