"""Golden vectors for the three-component eviction selection, produced by the reference's
own ThreeComponentEvictionPolicy.select_indices (cab_attention/eviction/policy.py), which
is plain torch and runs on the CPU. The module is loaded from the reference checkout by
file path.

    python tests/golden/make_evict_golden.py <reference root> [output.npz]
"""

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]

# (name, cache_len, keep_size, local, bridge, importance length or 0, attention?, seed)
CASES = [
    ("median_1000", 1000, 100, 0.3, 0.2, 1000, False, 1),
    ("median_short_imp", 777, 200, 0.25, 0.25, 500, False, 2),
    ("median_long_imp", 300, 64, 0.3, 0.2, 400, False, 3),
    ("attention_512", 512, 96, 0.3, 0.2, 512, True, 4),
    ("positional_no_scores", 400, 90, 0.3, 0.2, 0, False, 5),
    ("keep_exceeds_len", 50, 80, 0.3, 0.2, 50, False, 6),
    ("no_bridge", 333, 100, 0.5, 0.0, 333, False, 7),
]


def main(ref_root: str, out_path: str):
    path = Path(ref_root) / "cab_attention" / "eviction" / "policy.py"
    spec = importlib.util.spec_from_file_location("ref_policy", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    data = {}
    for name, L, K, lr, br, n_imp, with_attn, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        imp = torch.rand(n_imp, generator=g) if n_imp else None
        attn = torch.softmax(torch.randn(L, L, generator=g) * 2, dim=-1) if with_attn else None
        policy = ref.ThreeComponentEvictionPolicy(ref.EvictionConfig(lr, br, 1.0 - lr - br))
        keep, diag = policy.select_indices(L, K, imp, attn, device="cpu")
        data[f"{name}/params"] = np.array([L, K, lr, br], dtype=np.float64)
        data[f"{name}/importance"] = imp.numpy() if imp is not None else np.zeros(0, np.float32)
        data[f"{name}/attention"] = attn.numpy() if attn is not None else np.zeros((0, 0), np.float32)
        data[f"{name}/keep"] = keep.numpy()
        data[f"{name}/counts"] = np.array([diag["keep_size"], diag["local_count"], diag["importance_count"],
                                           diag["bridge_count"]], dtype=np.int64)
        print(name, len(keep), data[f"{name}/counts"])
    np.savez_compressed(out_path, names=np.array([c[0] for c in CASES]), **data)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else str(REPO / "tests" / "golden" / "evict_select.npz"))
