"""Golden vectors for the flash-attention-with-cumulative-scores path, produced by the
reference's own Triton kernel (``cab_attention/kernels/flash_attention_accumulate.py``,
``flash_attention_with_cumulative_scores``) as installed under ``baseline/_ref``.

The kernel is Triton, so this script needs a CUDA GPU (it is run once on a B200 box and
its output committed as ``tests/golden/flash_cumulative.npz``). The reference module is
loaded from its file path so that this repository's own ``cab_attention`` package cannot
shadow it.

    python tests/golden/make_flash_golden.py [output.npz]
"""

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
REF = REPO / "baseline" / "_ref" / "cab_attention" / "kernels" / "flash_attention_accumulate.py"

# (name, dtype, B, H, Nq, Nk, D, seed, initial cumulative length or 0)
CASES = [
    ("self_f16_d64", torch.float16, 1, 2, 300, 300, 64, 1, 0),
    ("self_bf16_d128", torch.bfloat16, 1, 2, 256, 256, 128, 2, 0),
    ("decode_f16_d128", torch.float16, 1, 2, 1, 261, 128, 3, 0),
    ("kvcache_bf16_d64", torch.bfloat16, 2, 1, 130, 515, 64, 4, 0),
    ("extend_f16_d64", torch.float16, 1, 2, 64, 200, 64, 5, 150),
]


def load_reference():
    spec = importlib.util.spec_from_file_location("ref_flash_attention_accumulate", REF)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(out_path: str):
    ref = load_reference()
    data = {}
    for name, dtype, B, H, Nq, Nk, D, seed, init_len in CASES:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(B, H, Nq, D, generator=g).to(dtype)
        k = torch.randn(B, H, Nk, D, generator=g).to(dtype)
        v = torch.randn(B, H, Nk, D, generator=g).to(dtype)
        init = torch.rand(B, H, init_len, generator=g) if init_len else None
        out, cum = ref.flash_attention_with_cumulative_scores(
            q.cuda(), k.cuda(), v.cuda(), None if init is None else init.cuda())
        torch.cuda.synchronize()
        data[f"{name}/q"] = q.float().numpy()
        data[f"{name}/k"] = k.float().numpy()
        data[f"{name}/v"] = v.float().numpy()
        data[f"{name}/dtype"] = np.array(str(dtype).replace("torch.", ""))
        data[f"{name}/init"] = init.numpy() if init is not None else np.zeros((B, H, 0), np.float32)
        data[f"{name}/out"] = out.float().cpu().numpy()
        data[f"{name}/cum"] = cum.float().cpu().numpy()
        print(name, tuple(out.shape), tuple(cum.shape), float(cum.sum()))
    np.savez_compressed(out_path, names=np.array([c[0] for c in CASES]), **data)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(REPO / "tests" / "golden" / "flash_cumulative.npz"))
