"""Strong (batch x head) sharding of one layer over 2 GPUs with NCCL (skipped with fewer
GPUs): each rank runs coarsen -> FRC -> top-k -> attention on its contiguous range of
(b, KV head) units, built from the per-slice seeds; the outputs, all-gathered, equal the
single-GPU layer bit for bit (every unit is computed independently of the others)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

B, HQ, HKV, N, D, SP = 2, 8, 4, 16384, 128, 0.95


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer(q, k, v):
    from cab_attention import CoarseCurvaturePredictor
    from cab_attention.kernels import block_sparse_attention
    idx, num = CoarseCurvaturePredictor(64, SP, 0.5).predict_blocks(q, k)
    return block_sparse_attention(q, k, v, idx, num, 64), idx


def _worker(rank, world, port, result):
    import torch.distributed as dist
    from datetime import timedelta
    from cab_attention import sharding, synthetic, _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        G = HQ // HKV
        s, e = sharding.unit_range(B * HKV, world, rank)
        units = [divmod(u, HKV) for u in range(s, e)]
        q, k, v = (t.cuda() for t in synthetic.make_unit_qkv(units, G, N, D, torch.bfloat16, 0))
        out, _ = _layer(q, k, v)
        full = torch.empty((world,) + tuple(out.shape[1:]), dtype=out.dtype, device=out.device)
        dist.all_gather_into_tensor(full, out)
        torch.cuda.synchronize()
        ok = _lib.device_status() == 0
        if rank == 0:
            qa, ka, va = (t.cuda() for t in synthetic.make_qkv(B, HQ, HKV, N, D, torch.bfloat16, 0))
            want, _ = _layer(qa, ka, va)
            got = full.view(B, HQ, N, D)
            result.put((ok, torch.equal(got, want), (got.float() - want.float()).abs().max().item()))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_strong_sharded_layer_equals_single_gpu():
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok, equal, err = result.get(timeout=5)
    assert ok and equal, err
