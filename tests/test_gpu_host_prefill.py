"""``prefill_from_host`` (``cab_prefill_host``): the streamed host-memory path must give
bit-identical results to the device path (predictor + block_sparse_attention on device
copies of the same tensors), for every unit count (slot reuse), GQA, causal and dtype."""

import pytest
import torch

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import CoarseCurvaturePredictor, _lib, prefill_from_host  # noqa: E402
from cab_attention.kernels import block_sparse_attention  # noqa: E402

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert _lib.device_status() == 0, "a kernel's bounded wait timed out"


def pinned(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).pin_memory()


@pytest.mark.parametrize("dt,B,Hq,Hkv,N,D,s,causal,norm", [
    ("bf16", 2, 4, 2, 3000, 128, 0.9, False, "abs"),     # GQA, 4 units (slots reused)
    ("bf16", 3, 1, 1, 5000, 128, 0.95, False, "abs"),    # 3 units, one head each
    ("f16", 1, 2, 2, 4096, 64, 0.8, True, "minmax"),     # causal, D=64
    ("bf16", 1, 1, 1, 777, 128, 0.5, False, "raw"),      # partial last block
    ("f32", 1, 2, 1, 1000, 64, 0.9, False, "abs"),       # CUDA-core kernels
])
def test_host_prefill_matches_device_path(dt, B, Hq, Hkv, N, D, s, causal, norm):
    q = pinned((B, Hq, N, D), DT[dt], 1)
    k = pinned((B, Hkv, N, D), DT[dt], 2)
    v = pinned((B, Hkv, N, D), DT[dt], 3)
    out, idx, num = prefill_from_host(q, k, v, sparsity=s, causal=causal, normalization=norm,
                                      return_indices=True)
    pred = CoarseCurvaturePredictor(block_size=64, sparsity=s, causal=causal,
                                    normalization=norm)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    ref_idx, ref_num = pred.predict_blocks(qd, kd)
    ref = block_sparse_attention(qd, kd, vd, ref_idx, ref_num, 64, causal)
    torch.cuda.synchronize()
    assert torch.equal(idx, ref_idx.cpu())
    assert torch.equal(num, ref_num.cpu())
    assert torch.equal(out, ref.cpu())


def test_host_prefill_into_given_out_async():
    q = pinned((1, 2, 2048, 128), torch.bfloat16, 4)
    k = pinned((1, 2, 2048, 128), torch.bfloat16, 5)
    v = pinned((1, 2, 2048, 128), torch.bfloat16, 6)
    out = torch.zeros_like(q).pin_memory()
    res = prefill_from_host(q, k, v, sparsity=0.75, out=out, synchronize=False)
    torch.cuda.current_stream().synchronize()
    assert res.data_ptr() == out.data_ptr()
    ref = prefill_from_host(q, k, v, sparsity=0.75)
    assert torch.equal(out, ref)


def test_host_prefill_rejects_pageable_and_device_inputs():
    q = torch.randn(1, 1, 256, 64).to(torch.bfloat16)
    with pytest.raises(ValueError, match="page-locked"):
        prefill_from_host(q, q, q)
    with pytest.raises(ValueError, match="CPU tensor"):
        prefill_from_host(q.cuda(), q.cuda(), q.cuda())
