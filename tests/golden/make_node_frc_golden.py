"""Golden vectors for node-level FRC from the reference's own ``compute_frc_pytorch``
(``cab_attention/kernels/frc_triton.py``), which runs on the CPU. The module is loaded
from the reference checkout by file path (it imports triton at module level, which loads
without a GPU).

    python tests/golden/make_node_frc_golden.py <reference root> [output.npz]
"""

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]


def main(ref_root: str, out_path: str):
    path = Path(ref_root) / "cab_attention" / "kernels" / "frc_triton.py"
    spec = importlib.util.spec_from_file_location("ref_frc_triton", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    data = {}
    names = []
    for name, N, seed, kind in (("rowstoch_100", 100, 1, "rowstoch"), ("rand_257", 257, 2, "rand"),
                                ("softmax_64", 64, 3, "softmax")):
        g = torch.Generator().manual_seed(seed)
        if kind == "rowstoch":
            a = torch.rand(N, N, generator=g)
            a = a / a.sum(dim=1, keepdim=True)
        elif kind == "rand":
            a = torch.rand(N, N, generator=g)
        else:
            a = torch.softmax(torch.randn(N, N, generator=g) * 3, dim=-1)
        frc = ref.compute_frc_pytorch(a)
        data[f"{name}/attention"] = a.numpy()
        data[f"{name}/frc"] = frc.numpy()
        names.append(name)
        print(name, float(frc.mean()))
    np.savez_compressed(out_path, names=np.array(names), **data)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else str(REPO / "tests" / "golden" / "node_frc.npz"))
