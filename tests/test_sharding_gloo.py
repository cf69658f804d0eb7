"""(batch x head) sharding on CPU ranks (gloo, world size 2): every unit is covered once,
shards built from per-(b,h) seeds equal slices of the whole batch, and the per-rank oracle
results gathered over the process group equal the single-process result."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cab_attention import sharding, synthetic


def test_unit_ranges_cover_everything_once():
    for units in (1, 7, 16, 32, 33):
        for world in (1, 2, 3, 4, 8):
            got = []
            for r in range(world):
                s, e = sharding.unit_range(units, world, r)
                got.extend(range(s, e))
            assert got == list(range(units))


def test_units_to_slices():
    assert sharding.units_to_slices(3, 11, 4) == [(0, 3, 4), (1, 0, 4), (2, 0, 3)]
    assert sharding.units_to_slices(0, 8, 8) == [(0, 0, 8)]


def test_shard_inputs_equal_whole_batch_slices():
    q, k, v = synthetic.make_qkv(4, 2, 2, 128, 16, torch.float32, seed=5)
    q2, k2, v2 = synthetic.make_qkv(2, 2, 2, 128, 16, torch.float32, seed=5, batch_offset=2)
    assert torch.equal(q[2:], q2) and torch.equal(k[2:], k2) and torch.equal(v[2:], v2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import cab_oracle as orc
        B, H, N, D, bs = 2, 3, 512, 16, 64
        units = B * H
        s, e = sharding.unit_range(units, world, rank)
        q, k, v = synthetic.make_qkv(B, H, H, N, D, torch.float32, seed=9)
        qs = q.reshape(units, 1, N, D)[s:e].permute(1, 0, 2, 3).numpy()
        ks = k.reshape(units, 1, N, D)[s:e].permute(1, 0, 2, 3).numpy()
        vs = v.reshape(units, 1, N, D)[s:e].permute(1, 0, 2, 3).numpy()
        o = orc.predictor(qs, ks, bs, 0.75, 0.5)
        out, _ = orc.block_sparse_attention(qs, ks, vs, o["kv_idx"], o["kv_num"], bs)
        local = torch.from_numpy(out[0])                       # [units_local, N, D]
        full = sharding.gather_units(local, units)
        result_q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_oracle_layer_equals_single_process():
    from oracle import cab_oracle as orc
    world = 2
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, result_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(result_q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    B, H, N, D, bs = 2, 3, 512, 16, 64
    q, k, v = synthetic.make_qkv(B, H, H, N, D, torch.float32, seed=9)
    o = orc.predictor(q.numpy(), k.numpy(), bs, 0.75, 0.5)
    want, _ = orc.block_sparse_attention(q.numpy(), k.numpy(), v.numpy(), o["kv_idx"],
                                         o["kv_num"], bs)
    want = want.reshape(B * H, N, D)
    for r in range(world):
        np.testing.assert_allclose(results[r], want, rtol=1e-12, atol=1e-12)


def _failing_worker(rank, world, port, result_q):
    """Rank 1 dies before the gather; rank 0's gather must end with an error (the process
    group timeout), not hang."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # the rank leaves between steps, with nothing of its own in flight
    try:
        sharding.gather_units(torch.zeros(1, 4), 2)
        result_q.put(("no error", rank))
    except Exception as e:  # noqa: BLE001 - the failure mode is what is tested
        result_q.put((type(e).__name__, rank))


def test_dead_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, rank = q.get(timeout=60)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and kind != "no error"


def test_unit_inputs_equal_whole_batch_slices():
    q, k, v = synthetic.make_qkv(2, 4, 2, 96, 8, torch.float32, seed=3)
    units = [(0, 1), (1, 0)]
    qu, ku, vu = synthetic.make_unit_qkv(units, 2, 96, 8, torch.float32, seed=3)
    assert torch.equal(qu[0, 0:2], q[0, 2:4]) and torch.equal(qu[0, 2:4], q[1, 0:2])
    assert torch.equal(ku[0, 0], k[0, 1]) and torch.equal(vu[0, 1], v[1, 0])


def test_bench_strong_plan_covers_units_evenly():
    """bench.py's strong-scaling plan (one layer's B x Hkv units over N ranks, two chunks per
    rank): every unit exactly once, equal shares where N divides the unit count, chunks that
    tile each rank's units."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    for name in ("ns", "c2", "c5"):
        cfg = bench.CONFIGS[name]
        n_units = cfg["B"] * cfg["Hkv"]
        for world in (2, 4, 8):
            seen = []
            for rank in range(world):
                lcfg, units, chunks = bench.shard_plan(cfg, rank, world, "strong")
                assert lcfg["Hkv"] == len(units) and lcfg["Hq"] == len(units) * (cfg["Hq"] // cfg["Hkv"])
                assert chunks[0][0] == 0 and chunks[-1][1] == len(units)
                assert all(a[1] == b[0] for a, b in zip(chunks, chunks[1:]))
                if n_units % world == 0:
                    assert len(units) == n_units // world
                seen += [b * cfg["Hkv"] + h for b, h in units]
            assert sorted(seen) == list(range(n_units))


def test_bench_peak_selection():
    """bench.py divides by the burst bf16 peak for a short timed window or a run at full
    clock, by the sustained one for a seconds-long window that settled under the power cap."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench_mod2", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    burst, sus = 1647.4, 1408.2
    assert bench.pick_peak({"sm_mhz": 1965.0, "sm_max_mhz": 1965.0}, 92.0, burst, sus)[0] == burst
    assert bench.pick_peak({"sm_mhz": 1600.0, "sm_max_mhz": 1965.0}, 500.0, burst, sus)[0] == burst
    assert bench.pick_peak({"sm_mhz": 1960.0, "sm_max_mhz": 1965.0}, 5000.0, burst, sus)[0] == burst
    assert bench.pick_peak({"sm_mhz": 1600.0, "sm_max_mhz": 1965.0}, 5000.0, burst, sus)[0] == sus
    assert bench.pick_peak({"sm_mhz": None, "sm_max_mhz": None}, 5000.0, burst, sus)[0] == sus
