"""Node-level FRC (cab_node_frc) against the float64 restatement and against the golden
vectors of the reference's own compute_frc_pytorch. Tolerance: 1e-5 of the largest |F|
for fp32 inputs; fp16/bf16 inputs are compared with the oracle evaluated on the same
(rounded) values, at 1e-4 (fp32 accumulation over N terms)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import _lib  # noqa: E402
from cab_attention.kernels.frc_triton import (compute_frc, compute_frc_pytorch,  # noqa: E402
                                              compute_frc_triton, compute_node_strengths_triton,
                                              compute_triangles_triton)

GOLDEN = Path(__file__).resolve().parent / "golden" / "node_frc.npz"


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert _lib.device_status() == 0


@pytest.mark.parametrize("dtype,shape", [(torch.float32, (100, 100)), (torch.float32, (1000, 1000)),
                                         (torch.float16, (2, 3, 257, 257)), (torch.bfloat16, (513, 513)),
                                         (torch.float32, (3, 4096, 4096))])
def test_node_frc_matches_oracle(dtype, shape):
    g = torch.Generator().manual_seed(shape[-1])
    a = torch.rand(*shape, generator=g)
    a = (a / a.sum(dim=-1, keepdim=True)).to(dtype)
    frc = compute_frc_triton(a.cuda())
    s = compute_node_strengths_triton(a.cuda())
    t = compute_triangles_triton(a.cuda())
    wf, ws, wt = orc.node_frc(a.float().numpy())
    tol = 1e-5 if dtype == torch.float32 else 1e-2  # outputs are rounded to the input dtype
    for got, want in ((frc, wf), (s, ws), (t, wt)):
        err = np.abs(got.double().cpu().numpy() - want).max() / max(1.0, np.abs(want).max())
        assert err <= tol, err
    assert frc.dtype == dtype
    assert torch.equal(compute_frc(a.cuda()), frc) and torch.equal(compute_frc_pytorch(a.cuda()), frc)


def test_node_frc_matches_reference_golden():
    g = np.load(GOLDEN)
    for name in g["names"]:
        a = torch.from_numpy(g[f"{name}/attention"]).cuda()
        ref = g[f"{name}/frc"].astype(np.float64)
        got = compute_frc(a).double().cpu().numpy()
        assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), name
