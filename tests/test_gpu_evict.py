"""Eviction selection (cab_evict_select) against the reference's own select_indices
(golden vectors) and the oracle restatement: kept index sets exact, counts exact."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import _lib  # noqa: E402
from cab_attention.eviction import (EvictionConfig, ThreeComponentEvictionPolicy,  # noqa: E402
                                    select_indices_batched)

GOLDEN = Path(__file__).resolve().parent / "golden" / "evict_select.npz"


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert _lib.device_status() == 0


def test_evict_matches_reference_golden():
    g = np.load(GOLDEN)
    for name in g["names"]:
        L, K, lr, br = g[f"{name}/params"]
        L, K = int(L), int(K)
        imp = g[f"{name}/importance"]
        att = g[f"{name}/attention"]
        policy = ThreeComponentEvictionPolicy(EvictionConfig(lr, br, 1.0 - lr - br))
        keep, diag = policy.select_indices(L, K, torch.from_numpy(imp).cuda() if imp.size else None,
                                           torch.from_numpy(att).cuda() if att.size else None)
        assert np.array_equal(keep.cpu().numpy(), g[f"{name}/keep"]), name
        counts = (diag["keep_size"], diag["local_count"], diag["importance_count"], diag["bridge_count"])
        assert counts == tuple(int(x) for x in g[f"{name}/counts"]), name


@pytest.mark.parametrize("L,K,n_imp,with_attn", [(131072, 8192, 131072, False), (4096, 1000, 3000, True),
                                                 (100000, 3, 100000, False), (70001, 20000, 0, False)])
def test_evict_batched_matches_oracle(L, K, n_imp, with_attn):
    g = torch.Generator().manual_seed(L + K)
    B = 3
    imp = torch.rand(B, n_imp, generator=g) if n_imp else None
    att = torch.softmax(torch.randn(B, L, L, generator=g), dim=-1) if with_attn else None
    keep, counts = select_indices_batched(L, K, imp.cuda() if imp is not None else None,
                                          att.cuda() if att is not None else None, 0.3, 0.2, batch=B)
    for b in range(B):
        wk, wc = orc.evict_select(L, K, imp[b].numpy() if imp is not None else None,
                                  att[b].numpy() if att is not None else None, 0.3, 0.2)
        n = int(counts[b, 0])
        assert tuple(int(x) for x in counts[b].tolist()) == tuple(wc)
        assert np.array_equal(keep[b, :n].cpu().numpy(), wk)
        assert (keep[b, n:] == -1).all()
