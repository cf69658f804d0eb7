"""The float32 torch CPU baseline (oracle/cab_torch_cpu.py, timed by bench.py) computes the
same layer as the float64 numpy oracle: block masks agree on >= 99.9 % of blocks and the
attention output matches to float32 precision given the same lists."""

import numpy as np
import torch

from oracle import cab_oracle as orc
from oracle import cab_torch_cpu as tcpu


def _case(N, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(N, D, generator=g).to(torch.bfloat16).float()
    k = torch.randn(N, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(N, D, generator=g).to(torch.bfloat16).float()
    return q, k, v


def test_predictor_matches_oracle():
    q, k, _ = _case(8192, 64, 3)
    idx, num = tcpu.predictor_head(q, k, 64, 0.9, 0.5)
    o = orc.predictor(q.numpy()[None, None], k.numpy()[None, None], 64, 0.9, 0.5)
    M = idx.shape[0]
    got = np.zeros((M, M), dtype=bool)
    got[np.arange(M)[:, None], idx.numpy()] = True
    assert (num == o["k"]).all()
    assert (got == o["mask"][0, 0]).mean() >= 0.999
    assert got[np.arange(M), np.arange(M)].all()  # diagonal kept


def test_attention_matches_oracle():
    q, k, v = _case(3000, 128, 4)          # partial last block
    M = (3000 + 63) // 64
    g = torch.Generator().manual_seed(5)
    idx = torch.stack([torch.randperm(M, generator=g)[:7].sort().values for _ in range(M)])
    got = tcpu.attention_head(q, k, v, idx, 64, chunk=5)
    want, _ = orc.block_sparse_attention(q.numpy()[None, None], k.numpy()[None, None], v.numpy()[None, None],
                                         idx.numpy()[None, None].astype(np.int32),
                                         np.full((1, 1, M), 7, dtype=np.int32), 64)
    assert np.abs(got.numpy() - want[0, 0]).max() <= 1e-4


def test_layer_timed_reports_extrapolation():
    q, k, v = (t[None, None].repeat(1, 2, 1, 1) for t in _case(2048, 64, 6))
    ms, info = tcpu.layer_timed(q, k, v, 64, 0.9, 0.5, budget_s=0.0)
    assert ms > 0 and info["heads"] == 2 and info["heads_measured"] == 1
    assert info["extrapolated"] and info["measured_fraction"] == 0.5
