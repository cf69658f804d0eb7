"""The prefill path under CUDA-graph capture: the predictor and the block-sparse attention
enqueue only stream-ordered work (no host synchronisation, allocations from the caller's
allocator), so torch.cuda.graph captures them; replaying the graph equals the eager call
bit for bit, and a replay after new data is copied into the captured input buffers equals
the eager call on that data."""

import pytest
import torch

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import CoarseCurvaturePredictor, _lib, synthetic  # noqa: E402
from cab_attention.kernels import block_sparse_attention  # noqa: E402


def test_cuda_graph_replay_matches_eager():
    q, k, v = (t.cuda() for t in synthetic.make_qkv(1, 4, 2, 8192, 128, torch.bfloat16, seed=5))
    pred = CoarseCurvaturePredictor(64, 0.9, 0.5)

    def layer():
        idx, num = pred.predict_blocks(q, k)
        return block_sparse_attention(q, k, v, idx, num, 64)

    eager = layer()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer()
    graph.replay()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(out, eager)

    q2, k2, v2 = synthetic.make_qkv(1, 4, 2, 8192, 128, torch.bfloat16, seed=6)
    q.copy_(q2)
    k.copy_(k2)
    v.copy_(v2)
    graph.replay()
    want = layer()
    torch.cuda.synchronize()
    assert not torch.equal(want, eager)
    assert torch.equal(out, want)
