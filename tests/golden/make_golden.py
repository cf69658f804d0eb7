"""Generate the golden fixtures in this folder by running the reference's own code.

Run in a container where the reference checkout is mounted (default ``/root/reference``,
or ``CAB_REFERENCE_DIR``); the GPU box never runs this. Outputs (small ``.npz`` files):

* ``test_ipynb_bridge.npz`` -- ``test.ipynb`` cell 0 executed as written (plots stubbed):
  the N=100 two-community adjacency, its augmented FRC matrix (bridge (0,99) = -85.71)
  and the H2O / CAB keep masks at every sparsity of the notebook.
* ``colab_v3_pipeline.npz`` -- ``CAB_Attention_Colab.ipynb`` cell 17
  ``run_cab_v3_pipeline`` executed on seeded fp32 inputs. The notebook imports
  ``coarsen_qk_max_l2`` from ``cab_attention/kernels/coarsening.py``, which the snapshot
  does not contain, so the oracle's Max-L2 coarsening is injected in its place; the
  fixture therefore pins everything downstream of coarsening (|A| FRC with lambda 0.5,
  global top-k threshold, token expansion, masked softmax, nan_to_num).
* ``methods_cabv3.npz`` -- ``experiments/longbench_qa/methods.py``
  ``CABV3Attention.modify_attention_weights`` (expand_block_mask + -inf masking + softmax
  + nan_to_num) on seeded causal logits, with the three missing stage functions bound to
  the oracle. It pins the reference's token-level expansion and masked-softmax semantics.

Usage: ``python tests/golden/make_golden.py``
"""

from __future__ import annotations

import importlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("CAB_REFERENCE_DIR", "/root/reference"))
sys.dont_write_bytecode = True
sys.path.insert(0, str(REPO))

from oracle import cab_oracle as orc  # noqa: E402


class _Anything:
    """Absorbs every plotting call of the notebooks (matplotlib/seaborn are absent)."""

    def __getattr__(self, name):
        return _Anything()

    def __call__(self, *a, **k):
        return _Anything()

    def __getitem__(self, k):
        return _Anything()

    def __iter__(self):
        return iter([_Anything(), _Anything()])


def _stub_plotting():
    for name in ("matplotlib", "matplotlib.pyplot", "seaborn"):
        mod = types.ModuleType(name)
        mod.__getattr__ = lambda attr: _Anything()
        sys.modules[name] = mod
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]

    def subplots(*a, **k):
        return _Anything(), _Anything()

    sys.modules["matplotlib.pyplot"].subplots = subplots


def _cell(nb_path, index):
    nb = json.loads(Path(nb_path).read_text())
    return "".join(nb["cells"][index]["source"])


def make_test_ipynb():
    _stub_plotting()
    ns = {"__name__": "__golden__"}
    exec(compile(_cell(REF / "test.ipynb", 0), "test.ipynb:cell0", "exec"), ns)
    adj = ns["adj"].cpu().numpy()
    frc = ns["compute_forman_ricci_curvature"](ns["adj"]).cpu().numpy()
    sparsities = [0.5, 0.8, 0.9, 0.95, 0.98, 0.99]
    h2o = np.stack([ns["get_topk_mask"](ns["adj"], s, largest=True).cpu().numpy()
                    for s in sparsities])
    cab = np.stack([ns["get_topk_mask"](torch.tensor(frc), s, largest=False).cpu().numpy()
                    for s in sparsities])
    np.savez_compressed(HERE / "test_ipynb_bridge.npz", adj=adj, frc=frc,
                        sparsities=np.array(sparsities), h2o_masks=h2o, cab_masks=cab,
                        bridge=np.array([0, 99]))
    print("test.ipynb: bridge FRC", frc[0, 99])


def _torch_coarsen(q, k, block_size=64):
    qc, _ = orc.coarsen_maxl2(q.detach().cpu().numpy(), block_size)
    kc, _ = orc.coarsen_maxl2(k.detach().cpu().numpy(), block_size)
    return torch.from_numpy(qc).to(q.dtype), torch.from_numpy(kc).to(k.dtype)


def make_colab_pipeline():
    ns = {"__name__": "__golden__", "torch": torch,
          "coarsen_qk_max_l2": _torch_coarsen}
    exec(compile(_cell(REF / "CAB_Attention_Colab.ipynb", 17), "colab:cell17", "exec"), ns)
    cases = {}
    for case, (B, H, N, D, bs, sp, seed) in enumerate([(1, 2, 256, 32, 32, 0.90, 11),
                                                        (2, 1, 200, 16, 32, 0.80, 12)]):
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, H, N, D, generator=g)
        k = torch.randn(B, H, N, D, generator=g)
        v = torch.randn(B, H, N, D, generator=g)
        out, stats = ns["run_cab_v3_pipeline"](q, k, v, sparsity=sp, block_size=bs)
        cases.update({f"c{case}_q": q.numpy(), f"c{case}_k": k.numpy(), f"c{case}_v": v.numpy(),
                      f"c{case}_out": out.numpy(),
                      f"c{case}_meta": np.array([bs, stats["blocks_kept"]], dtype=np.float64),
                      f"c{case}_sparsity": np.array(sp)})
    np.savez_compressed(HERE / "colab_v3_pipeline.npz", **cases)
    print("colab pipeline cases:", len(cases) // 6)


def make_methods_cabv3():
    sys.path.insert(0, str(REF))
    methods = importlib.import_module("experiments.longbench_qa.methods")
    config = importlib.import_module("experiments.longbench_qa.config")
    cfg = config.MethodConfig(name="cab", sparsity=0.75, block_size=16, lambda_redundancy=0.5,
                              formula="additive", normalization="abs", causal=True,
                              keep_diagonal=True)
    m = methods.CABV3Attention(cfg)

    def frc_fn(qc, kc, temperature=1.0, lambda_redundancy=0.5, formula="additive",
               normalization="abs"):
        f, a, r = orc.block_frc(qc.numpy(), kc.numpy(), temperature, lambda_redundancy,
                                normalization, formula)
        return torch.from_numpy(f), torch.from_numpy(a), torch.from_numpy(r)

    def mask_fn(frc, sparsity, select_high=True, keep_diagonal=True, causal=False):
        M = frc.shape[-1]
        _, _, dense = orc.topk_block_mask(frc.numpy(), orc.keep_count(M, sparsity),
                                          select_high, keep_diagonal, causal)
        return torch.from_numpy(dense)

    m.coarsen_fn = _torch_coarsen
    m.frc_fn = frc_fn
    m.mask_fn = mask_fn
    m._cab_available = True
    g = torch.Generator().manual_seed(21)
    B, H, N, D = 1, 2, 120, 16
    q = torch.randn(B, H, N, D, generator=g)
    k = torch.randn(B, H, N, D, generator=g)
    logits = (q @ k.transpose(-1, -2)) / D ** 0.5
    causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
    logits = logits.masked_fill(~causal, float("-inf"))
    w, diag = m.modify_attention_weights(logits, q, k)
    np.savez_compressed(HERE / "methods_cabv3.npz", q=q.numpy(), k=k.numpy(),
                        logits=logits.numpy(), weights=w.numpy(),
                        params=np.array([16, 0.75, 0.5]))
    print("methods CABV3: sparsity", diag["sparsity"])


if __name__ == "__main__":
    torch.set_num_threads(1)
    make_test_ipynb()
    make_colab_pipeline()
    make_methods_cabv3()
