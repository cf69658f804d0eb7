"""Benchmark of the CAB prefill layer (predictor + block-sparse attention) on B200.

Metric: "CAB layer ms @N=128k (predictor + sparse attn)". Default workload:
the north_star shape B=2, H=8, N=128000, D=128, bf16, block 64, sparsity 0.95 (k=100 of
M=2000 key blocks per row), lambda 0.5, |A| FRC, highest-F selection with the diagonal
kept, non-causal. Q, K, V iid N(0,1) from per-(b,h) seeded generators (synthetic data,
the reference measures on random tensors too).

One step = Max-L2 coarsening -> FRC (two tensor-core GEMMs) -> per-row top-k -> pair-union
lists -> block-sparse attention. Multi-GPU (one process per GPU, torchrun): by default the
layer's B x Hkv (batch, KV head) units are split over the ranks (strong scaling; the
north_star partition), each rank computes its units in two chunks and all-gathers each
chunk's output over NCCL on a side stream inside the timed region; ``value`` = the
max-over-ranks layer latency. ``--scaling weak`` gives every rank its own whole layer
instead (``value`` = step time / world, ms per layer-equivalent).

``--impl reference`` times the reference's path on the host CPU: the reference's own
implementation of this path is absent from its snapshot, so its CPU restatement under
oracle/ (float32 torch on all host threads, oracle/cab_torch_cpu.py) is timed on whole
(b, h) heads within a per-step budget and extrapolated per head.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "bridge-aware-kv-cache-eviction-for-efficient-long-context-transformers_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

CONFIGS = {
    "ns": dict(B=2, Hq=8, Hkv=8, N=128000, D=128, sparsity=0.95, causal=False,
               workload="north_star CAB layer: B2 H8 N128000 D128 bf16, block 64, s=0.95 (k=100/M=2000)"),
    "c2": dict(B=2, Hq=8, Hkv=8, N=32768, D=128, sparsity=0.95, causal=False,
               workload="configs[1]: B2 H8 N32768 D128 bf16, block 64, s=0.95"),
    "c5": dict(B=1, Hq=32, Hkv=8, N=65536, D=128, sparsity=0.99, causal=True,
               workload="configs[4]: GQA 32/8 B1 N65536 D128 bf16 causal, s=0.99"),
    # the reference's live flash kernel with cumulative column scores (next-row scope)
    # node-level FRC of attention graphs and the eviction selection (next-row scope)
    "nodefrc": dict(B=16, Hq=1, Hkv=1, N=4096, D=0, sparsity=0.0, causal=False,
                    workload="node-level FRC: 16 row-stochastic fp32 attention graphs of 4096 nodes "
                             "(compute_frc)"),
    "evict": dict(B=32, Hq=1, Hkv=1, N=131072, D=8192, sparsity=0.0, causal=False,
                  workload="eviction selection: 32 caches of 131072 tokens, keep 8192 "
                           "(local 0.3 / bridge 0.2 / importance 0.5, median bridges; select_indices)"),
    "flash": dict(B=1, Hq=8, Hkv=8, N=32768, D=128, sparsity=0.0, causal=False,
                  workload="flash attention + cumulative column scores: B1 H8 N32768 D128 bf16, "
                           "non-causal (flash_attention_with_cumulative_scores)"),
    # the CABAttention layer at the README scale (D = dim / heads = 64)
    "c3": dict(B=2, Hq=8, Hkv=8, N=128000, D=64, dim=512, sparsity=0.95, causal=False,
               workload="configs[2]: CABAttention(dim=512, heads=8, head_dim=64) B2 N128000 bf16, s=0.95, "
                        "projection weights N(0, 0.02^2)"),
    # predictor-only latency per N (the line's value is the largest N)
    "sweep": dict(B=2, Hq=8, Hkv=8, N=131072, D=128, sparsity=0.95, causal=False,
                  workload="configs[3]: CoarseCurvaturePredictor over N in {1k, 4k, 16k, 64k, 128k}, "
                           "B2 H8 D128 bf16, s=0.95"),
}
SWEEP_N = (1024, 4096, 16384, 65536, 131072)
BLOCK = 64
LAMBDA = 0.5


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of this rank's GPU, read every
    10 ms through NVML on a background thread (read-only queries); only the samples taken
    between mark_start() and mark_end() -- wall clock around the synchronised timed
    region -- are reported. Without NVML it falls back to nvidia-smi at 200 ms."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        self.rank_dev = local_rank
        self.samples = []  # (t, sm_mhz, reason bits or names, power_w)
        self.t0 = self.t1 = None
        self.max_mhz = None
        self.proc = None
        self.stop_flag = threading.Event()
        self.thread = None
        self.mode = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.rank_dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.rank_dev)

    def start(self):
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.mode = "nvml"

            def loop():
                while not self.stop_flag.is_set():
                    try:
                        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                        pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                        self.samples.append((time.monotonic(), sm, rs, pw))
                    except Exception:
                        pass
                    time.sleep(0.01)
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.mode = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.rank_dev)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.mode = "nvidia-smi"

            def read():
                names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
                for line in self.proc.stdout:
                    parts = [x.strip() for x in line.strip().split(",")]
                    if len(parts) < 8:
                        continue
                    try:
                        sm, mx = float(parts[0]), float(parts[1])
                    except ValueError:
                        continue
                    self.max_mhz = mx
                    rs = {n for n, v in zip(names, parts[4:8]) if v.lower().startswith("active")}
                    self.samples.append((time.monotonic(), sm, rs, None))
            self.thread = threading.Thread(target=read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def stop(self):
        if self.mode is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        win = [x for x in list(self.samples) if t0 <= x[0] <= t1]
        reasons = set()
        for _, _, rs, _ in win:
            if isinstance(rs, int):
                reasons |= {n for n, bit in self.REASONS if rs & bit}
            else:
                reasons |= rs
        pw = [x[3] for x in win if x[3] is not None]
        out = {"sm_mhz": statistics.median(x[1] for x in win) if win else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(reasons), "samples": len(win), "source": self.mode}
        if pw:
            out["power_w_median"] = round(statistics.median(pw), 1)
        return out


# --------------------------------------------------------------------------- our arm
def make_inputs(cfg, rank, seed, pin):
    from cab_attention import synthetic
    return synthetic.make_qkv(cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["N"], cfg["D"], torch.bfloat16,
                              seed, batch_offset=rank * cfg["B"], pin=pin)


class Layer:
    """One CAB layer step on device-resident q, k, v; every stage is one C-ABI call."""

    def __init__(self, cfg):
        from cab_attention import CoarseCurvaturePredictor
        self.cfg = cfg
        self.pred = CoarseCurvaturePredictor(block_size=BLOCK, sparsity=cfg["sparsity"],
                                             lambda_redundancy=LAMBDA, causal=cfg["causal"])

    def stages(self, q, k, v, events=None):
        from cab_attention.kernels import (block_sparse_attention, coarsen_qk_max_l2,
                                           compute_block_frc, topk_blocks)
        ev = events
        if ev: ev[0].record()
        qc, kc = coarsen_qk_max_l2(q, k, BLOCK)
        if ev: ev[1].record()
        frc, _, _ = compute_block_frc(qc, kc, 1.0, LAMBDA, return_affinity=False,
                                      return_redundancy=False)
        if ev: ev[2].record()
        kv_idx, kv_num, _ = topk_blocks(frc, self.pred.keep_per_row(q.shape[2]), True, True,
                                        self.cfg["causal"], return_dense=False)
        if ev: ev[3].record()
        out = block_sparse_attention(q, k, v, kv_idx, kv_num, BLOCK, self.cfg["causal"])
        if ev: ev[4].record()
        return out, kv_idx, kv_num

    def e2e(self, q_host, k_host, v_host, out_host):
        """Public-API call with host buffers (cab_prefill_host): the pinned inputs are
        copied in and the output copied back inside the call, streamed per (b, KV head)
        unit so the copies overlap the compute; returns after the output has landed."""
        from cab_attention import prefill_from_host
        prefill_from_host(q_host, k_host, v_host, block_size=BLOCK, sparsity=self.cfg["sparsity"],
                          lambda_redundancy=LAMBDA, causal=self.cfg["causal"], out=out_host)


_CPU_INPUTS = {}  # the CPU baseline's inputs, made once per run (not part of a timed step)


def cpu_sample(cfg, seconds_budget, seed=0):
    """The reference path on the host CPU, on a bounded sample of the workload, extrapolated
    to one layer. Non-causal configurations: the float32 torch restatement
    (oracle/cab_torch_cpu.py) on all host threads -- the predictor of every head in full,
    attention head by head until the budget is spent. Causal ones: the float64
    numpy oracle on one head's predictor and a sample of its query blocks.
    Returns (ms per layer, cpu_baseline dict without the value)."""
    from oracle import cab_torch_cpu as tcpu
    from cab_attention import synthetic
    torch.set_num_threads(os.cpu_count())
    N, D = cfg["N"], cfg["D"]
    base = {"unit": "ms", "cores": torch.get_num_threads(), "cpu_model": tcpu.cpu_model(), "kind": "port"}
    if not cfg["causal"]:
        key = (cfg["B"], cfg["Hq"], cfg["Hkv"], N, D, seed)
        if key not in _CPU_INPUTS:
            _CPU_INPUTS.clear()
            _CPU_INPUTS[key] = synthetic.make_qkv(cfg["B"], cfg["Hq"], cfg["Hkv"], N, D, torch.bfloat16, seed)
        q, k, v = _CPU_INPUTS[key]
        ms, info = tcpu.layer_timed(q, k, v, BLOCK, cfg["sparsity"], LAMBDA, budget_s=seconds_budget)
        heads = info["heads"]
        desc = (f"float32 torch on {base['cores']} threads: {info['heads_measured']} of {heads} (b, h) heads in "
                f"full (predictor, then attention over the kept K/V blocks gathered and multiplied with "
                f"bmm), {ms * info['measured_fraction'] / 1e3:.1f} s measured"
                + (", extrapolated linearly to every head" if info["extrapolated"] else ""))
        return ms, dict(base, dtype="f32", sample=desc, extrapolated=info["extrapolated"],
                        measured_fraction=round(info["measured_fraction"], 4),
                        predictor_ms=round(info["predictor_ms"], 1), attention_ms=round(info["attention_ms"], 1))
    from oracle import cab_oracle as orc
    M = (N + BLOCK - 1) // BLOCK
    q = synthetic.normal_heads("q", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    k = synthetic.normal_heads("k", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    v = synthetic.normal_heads("v", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    kk = orc.keep_count(M, cfg["sparsity"])
    t0 = time.perf_counter()
    qc, _ = orc.coarsen_maxl2(q, BLOCK)
    kc, _ = orc.coarsen_maxl2(k, BLOCK)
    t1 = time.perf_counter()
    frc, _, _ = orc.block_frc(qc, kc, 1.0, LAMBDA, "abs")
    idx, num, _ = orc.topk_block_mask(frc, kk, True, True, cfg["causal"])
    t3 = time.perf_counter()
    nb = 1
    while True:
        rows = [(0, 0, i) for i in range(0, M, max(1, M // nb))][:nb]
        s = time.perf_counter()
        orc.block_sparse_attention(q, k, v, idx, num, BLOCK, cfg["causal"], rows=rows)
        ta = time.perf_counter() - s
        if ta > seconds_budget * 0.3 or nb >= M or (t3 - t0) + ta > seconds_budget:
            break
        nb = min(M, nb * 4)
    heads = cfg["B"] * cfg["Hq"]
    coarsen_ms = (t1 - t0) * 1e3 * cfg["B"] * (cfg["Hq"] + cfg["Hkv"]) / 2.0
    pred_ms = coarsen_ms + (t3 - t1) * 1e3 * heads
    attn_ms = ta * 1e3 / len(rows) * M * heads
    desc = (f"float64 numpy oracle: predictor of 1 of {heads} heads at full N={N} "
            f"({(t3 - t0):.1f} s) + attention of {len(rows)} of {M} query blocks of that head "
            f"({ta:.1f} s), extrapolated linearly to the whole layer")
    measured = (t3 - t0) * 1e3 + ta * 1e3
    return pred_ms + attn_ms, dict(base, dtype="f64", sample=desc, extrapolated=True,
                                   measured_fraction=round(measured / (pred_ms + attn_ms), 6))


def pick_peak(clocks, window_ms, tf_burst, tf_sus):
    """Burst peak for a short timed window at full clock (the driver's runs), sustained for
    a window long enough to settle under the power cap."""
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if window_ms < 1000.0 or (sm and mx and sm >= 0.95 * mx):
        return tf_burst, "bf16_tflops (burst: timed window %.0f ms, median SM clock %s of max %s MHz)" % (
            window_ms, sm, mx)
    return tf_sus, "bf16_tflops_sustained (timed window %.0f ms under the power cap, SM clock %s MHz)" % (
        window_ms, sm)


def shard_plan(cfg, rank, world, scaling):
    """(local config, unit list, chunks). Strong scaling: the layer's B x Hkv (batch, KV
    head) units are split into contiguous ranges (cab_attention.sharding.unit_range) and the
    rank's units packed as one batch of heads; weak: every rank runs a whole layer on its
    own batch slice."""
    from cab_attention import sharding
    G = cfg["Hq"] // cfg["Hkv"]
    if world == 1 or scaling == "weak":
        return dict(cfg), None, [(0, cfg["Hkv"])]
    s, e = sharding.unit_range(cfg["B"] * cfg["Hkv"], world, rank)
    units = [divmod(u, cfg["Hkv"]) for u in range(s, e)]
    n = len(units)
    lcfg = dict(cfg, B=1, Hq=n * G, Hkv=n)
    nch = min(2, n)  # two chunks: the gather of the first overlaps the compute of the second
    cuts = [round(i * n / nch) for i in range(nch + 1)]
    return lcfg, units, [(cuts[i], cuts[i + 1]) for i in range(nch)]


def run_ours(args, cfg, rank, world, local_rank):
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    from cab_attention import _lib, synthetic
    from cab_attention.kernels.sparse_attention import sparse_attention_flops
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    scaling = args.scaling if world > 1 else "strong"
    lcfg, units, chunks = shard_plan(cfg, rank, world, scaling)
    G = cfg["Hq"] // cfg["Hkv"]
    if units is None:
        q_h, k_h, v_h = make_inputs(cfg, rank if scaling == "weak" else 0, args.seed, pin=True)
    else:
        q_h, k_h, v_h = synthetic.make_unit_qkv(units, G, cfg["N"], cfg["D"], torch.bfloat16, args.seed, pin=True)
    q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    out_h = torch.empty_like(q_h).pin_memory()
    layer = Layer(lcfg)
    strong = scaling == "strong" and world > 1
    side = torch.cuda.Stream(device=dev)
    # gathered output, chunk-major: gbuf[c] holds chunk c of every rank ([world, heads of
    # chunk c, N, D]); the whole [B, Hq, N, D] is a strided view of these buffers
    gbuf = [torch.empty((world, (c1 - c0) * G) + tuple(q.shape[2:]), dtype=q.dtype, device=dev)
            for (c0, c1) in chunks] if strong else []

    def step(evs=None):
        works, kv_num = [], []
        for ci, (c0, c1) in enumerate(chunks):
            qc, kc, vc = q[:, c0 * G:c1 * G], k[:, c0:c1], v[:, c0:c1]
            out_c, _, num_c = layer.stages(qc, kc, vc, evs[ci] if evs else None)
            kv_num.append(num_c)
            if strong:
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    works.append(dist.all_gather_into_tensor(gbuf[ci], out_c, async_op=True))
                out_c.record_stream(side)
        for w in works:
            w.wait()
        return kv_num

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # warm-up
    for _ in range(args.warmup):
        kv_num = step()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    # ---- timed region: device-resident inputs (inputs 1.5 GB per layer > 126 MB L2)
    nstage = 5
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(nstage)] for _ in chunks]
           for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    barrier()
    sampler.mark_start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for s in range(args.steps):
        kv_num = step(evs[s])
    end.record()
    barrier()
    sampler.mark_end()
    clocks = sampler.stop()
    total_ms = start.elapsed_time(end)
    stage_ms = np.array([[sum(evs[s][c][i].elapsed_time(evs[s][c][i + 1]) for c in range(len(chunks)))
                          for i in range(nstage - 1)] for s in range(args.steps)]).mean(axis=0)
    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = t.item() / args.steps
    assert _lib.device_status() == 0

    # ---- the gather alone (strong scaling): every chunk's all-gather without the compute
    gather_ms = None
    if strong:
        locs = [torch.empty_like(g[0]) for g in gbuf]
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            for ci in range(len(chunks)):
                dist.all_gather_into_tensor(gbuf[ci], locs[ci])
        g1.record()
        barrier()
        tg = torch.tensor([g0.elapsed_time(g1) / args.steps], device=dev, dtype=torch.float64)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        gather_ms = tg.item()

    # ---- end to end through the public API with host buffers (each rank its own units)
    for _ in range(max(1, args.warmup // 2)):
        layer.e2e(q_h, k_h, v_h, out_h)
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        layer.e2e(q_h, k_h, v_h, out_h)
    e_end.record()
    barrier()
    te = torch.tensor([e_start.elapsed_time(e_end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_step_ms = te.item() / args.steps

    # ---- roofline of each stage (algorithmic work of this rank / its measured time)
    B, Hq, Hkv, N, D = lcfg["B"], lcfg["Hq"], lcfg["Hkv"], lcfg["N"], lcfg["D"]
    M = (N + BLOCK - 1) // BLOCK
    kk = layer.pred.keep_per_row(N)
    from cab_attention import roofline as rl
    coarsen_bytes = rl.coarsen_bytes(B, Hq, Hkv, N, D, 2, BLOCK)
    frc_flop = rl.frc_flops(B, Hq, M, D)
    topk_bytes = rl.topk_bytes(B, Hq, M, kk)
    attn_flop = sum(sparse_attention_flops(n, BLOCK, D) for n in kv_num)
    kept = int(sum(int(n.sum().item()) for n in kv_num))
    c_ms, f_ms, k_ms, a_ms = (float(x) for x in stage_ms)
    peak, peak_src = pick_peak(clocks, total_ms, tf_burst, tf_sus)
    stages = {
        "coarsen": {"ms": c_ms, "GB/s": coarsen_bytes / c_ms / 1e6, "frac_hbm": coarsen_bytes / c_ms / 1e6 / hbm},
        "frc": {"ms": f_ms, "TFLOP/s": frc_flop / f_ms / 1e9, "frac_bf16": frc_flop / f_ms / 1e9 / peak},
        "topk": {"ms": k_ms, "GB/s": topk_bytes / k_ms / 1e6, "frac_hbm": topk_bytes / k_ms / 1e6 / hbm},
        "attention": {"ms": a_ms, "TFLOP/s": attn_flop / a_ms / 1e9, "frac_bf16": attn_flop / a_ms / 1e9 / peak,
                      "frac_bf16_sustained": attn_flop / a_ms / 1e9 / tf_sus, "kept_block_pairs": kept},
    }
    achieved = attn_flop / a_ms / 1e9
    roofline = {"bound": "tensor", "kernel": "attn_tc_kernel (block-sparse attention)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{peak_kind} {peak_src}",
                "frac_of_sustained": achieved / tf_sus,
                "traffic": ATTN_TRAFFIC_BYTES.get(args.config) if world == 1 else None}

    # ---- the reference's GPU attention step on the same inputs and lists: FlexAttention
    flex = None
    if world == 1 and args.flex and len(chunks) == 1:
        flex = flex_compare(q, k, v, layer, lcfg, args, peak)

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and args.cpu_baseline_seconds > 0:
            ms, info = cpu_sample(cfg, args.cpu_baseline_seconds, args.seed)
            cpu = dict(info, value=ms)
        h2d = world * sum(x.numel() * x.element_size() for x in (q_h, k_h, v_h))
        d2h = world * out_h.numel() * out_h.element_size()
        launches_per_step = 6 * len(chunks)  # coarsen, affinity GEMM, triangle GEMM, top-k, pair-union, attention
        if strong:
            par = (f"(batch x head) strong scaling: the layer's {cfg['B'] * cfg['Hkv']} (b, KV head) units split "
                   f"over {world} ranks ({len(units)} per rank, {len(chunks)} chunks); each chunk's output "
                   f"all-gathered over NCCL inside the timed region on a side stream")
        elif world > 1:
            par = f"weak scaling: every rank runs its own whole layer (global batch {cfg['B'] * world}), no collective"
        else:
            par = "one GPU, no collective"
        result = {
            "metric": "CAB layer ms @N=128k (predictor + sparse attn)",
            "value": step_ms if (strong or world == 1) else step_ms / world,
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": False,
            "scaling": "strong" if (strong or world == 1) else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K/V)",
            "config": {"workload": cfg["workload"], "layers_per_step": 1 if (strong or world == 1) else world,
                       "per_rank": f"B={B} Hq={Hq} Hkv={Hkv} N={N} D={D}",
                       "parallelism": par,
                       "l2": "inputs 1.5 GB per layer > 126 MB L2; no flush needed"},
            "stages": stages,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_step_ms if (strong or world == 1) else e2e_step_ms / world, "unit": "ms",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        if flex is not None:
            result["flex"] = flex
            if "ms" in flex:
                result["flex_ms"] = flex["ms"]
        if gather_ms is not None:
            result["gather_ms"] = gather_ms
            result["gather_bytes_per_rank"] = sum(g.numel() * g.element_size() for g in gbuf)
    return result


def flex_compare(q, k, v, layer, lcfg, args, peak):
    """Times torch's FlexAttention (compiled) on the same inputs and the same kept-block
    lists (oracle/flex_reference.py), for the same-box bar beside attn_tc_kernel."""
    try:
        from oracle import flex_reference as fr
        from cab_attention.kernels import block_sparse_attention
        from cab_attention.kernels.sparse_attention import sparse_attention_flops
        out, kv_idx, kv_num = layer.stages(q, k, v)
        bm = fr.block_mask(kv_idx, kv_num, lcfg["N"], BLOCK, lcfg["causal"])
        t0 = time.perf_counter()
        ref = fr.attention(q, k, v, bm)
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        diff = (ref.float() - out.float()).abs().max().item()
        del ref
        for _ in range(2):
            fr.attention(q, k, v, bm)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        o0, o1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            fr.attention(q, k, v, bm)
        e1.record()
        o0.record()
        for _ in range(args.steps):
            block_sparse_attention(q, k, v, kv_idx, kv_num, BLOCK, lcfg["causal"])
        o1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        ours_ms = o0.elapsed_time(o1) / args.steps
        flop = sparse_attention_flops(kv_num, BLOCK, lcfg["D"])
        return {"ms": ms, "TFLOP/s": flop / ms / 1e9, "frac_bf16": flop / ms / 1e9 / peak,
                "ours_ms_same_loop": ours_ms, "speedup_ours": ms / ours_ms,
                "max_abs_diff_vs_ours": diff, "compile_s": round(compile_s, 1),
                "what": f"torch {torch.__version__} flex_attention (torch.compile), BlockMask.from_kv_blocks "
                        f"BLOCK_SIZE={BLOCK} from the same kv_idx / kv_num, kept blocks as full blocks"}
    except Exception as e:  # the comparison must not take the benchmark down
        return {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}


# dram__bytes_read.sum + dram__bytes_write.sum per attention launch, from ncu captures of
# attn_tc_kernel<128, bf16, sparse> on the north_star shape with 4 of its 16 (b, h) units
# (401.845 MB read + 108.673 MB written) and of attn_tc_kernel<64, bf16, sparse> in the
# configs[2] layer with 1 of its 2 batches (478.420 MB read + 108.516 MB written). DRAM
# traffic is per unit (each unit reads its own Q/K/V once and writes its own O), so the
# full launches are scaled by 16 / 4 and by 2.
ATTN_TRAFFIC_BYTES = {"ns": (401.845248e6 + 108.672768e6) * 4,
                      "c3": (478.419712e6 + 108.515840e6) * 2}


# --------------------------------------------------------------------------- reference arm
def run_reference(args, cfg, sampler=None, metric="CAB layer ms @N=128k (predictor + sparse attn)"):
    """The reference path's CPU restatement on the host cores (all threads), a bounded
    sample per step (cpu_sample)."""
    sampler = sampler or cpu_sample
    budget = max(2.0, args.reference_step_seconds)
    for _ in range(args.warmup):
        sampler(cfg, budget, args.seed)
    vals, info = [], {}
    for _ in range(args.steps):
        ms, info = sampler(cfg, budget, args.seed)
        vals.append(ms)
    value = statistics.median(vals)
    return {
        "metric": metric,
        "impl": "reference",
        "value": value,
        "unit": "ms",
        "n_gpus": 0,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": value,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": info.get("dtype", "f32"),
        "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K/V)",
        "config": {"workload": cfg["workload"]},
        "cpu_baseline": dict(info, value=value),
        "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference snapshot lacks this path's implementation (its coarse_predictor / "
                 "cab_attention / kernels modules are listed in its README but absent), so its "
                 "CPU restatement under oracle/ is timed"),
    }


# --------------------------------------------------------------------------- CABAttention layer
def _c3_layer(cfg, seed, dev):
    from cab_attention import CABAttention
    layer = CABAttention(cfg["dim"], cfg["Hq"], block_size=BLOCK, sparsity=cfg["sparsity"],
                         lambda_redundancy=LAMBDA)
    layer.reset_parameters(torch.Generator().manual_seed(seed + 1))
    return layer.to(torch.bfloat16).to(dev)


def _c3_input(cfg, seed, rank, pin):
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    x = torch.randn(cfg["B"], cfg["N"], cfg["dim"], generator=g).to(torch.bfloat16)
    return x.pin_memory() if pin else x


def run_c3_ours(args, cfg, rank, world, local_rank):
    """CABAttention forward (fused QKV projection, predictor, block-sparse
    attention into the [B, N, dim] layout, output projection) on a device-resident x."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    from cab_attention import _lib
    from cab_attention.kernels import block_sparse_attention
    from cab_attention.kernels.sparse_attention import sparse_attention_flops
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    B, N, dim, H, D = cfg["B"], cfg["N"], cfg["dim"], cfg["Hq"], cfg["D"]
    layer = _c3_layer(cfg, args.seed, dev)
    x_h = _c3_input(cfg, args.seed, rank, pin=True)
    x = x_h.to(dev)
    out_h = torch.empty(B, N, dim, dtype=torch.bfloat16).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def staged(ev):
        ev[0].record()
        qkv = layer.qkv(x)
        q, k, v = layer.split_heads(qkv)
        ev[1].record()
        idx, num = layer.predictor.predict_blocks(q, k)
        ev[2].record()
        ctx = torch.empty(B, N, dim, dtype=x.dtype, device=dev)
        block_sparse_attention(q, k, v, idx, num, BLOCK, out=ctx.view(B, N, H, D).transpose(1, 2))
        ev[3].record()
        out = layer.proj(ctx)
        ev[4].record()
        return out, num

    with torch.no_grad():
        for _ in range(args.warmup):
            layer(x)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        sampler = ClockSampler(local_rank)
        sampler.start()
        time.sleep(0.2)
        barrier()
        sampler.mark_start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            layer(x)
        end.record()
        barrier()
        sampler.mark_end()
        clocks = sampler.stop()
        t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = t.item() / args.steps
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
        for st in range(args.steps):
            _, num = staged(evs[st])
        torch.cuda.synchronize()
        st_ms = [statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps))
                 for j in range(4)]
        # end to end through the module with host buffers: x in, out back, every step
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            out_h.copy_(layer(x_h.to(dev, non_blocking=True)), non_blocking=True)
        e1.record()
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
    attn_flop = sparse_attention_flops(num, BLOCK, D)
    proj_flop = 2.0 * B * N * dim * 3 * dim
    out_flop = 2.0 * B * N * dim * dim
    achieved = attn_flop / st_ms[2] / 1e9
    peak, peak_src = pick_peak(clocks, step_ms * args.steps, tf_burst, tf_sus)
    stages = {
        "qkv_proj": {"ms": st_ms[0], "TFLOP/s": proj_flop / st_ms[0] / 1e9},
        "predictor": {"ms": st_ms[1]},
        "attention": {"ms": st_ms[2], "TFLOP/s": achieved, "frac_bf16": achieved / peak,
                      "kept_block_pairs": int(num.sum().item())},
        "out_proj": {"ms": st_ms[3], "TFLOP/s": out_flop / st_ms[3] / 1e9},
    }
    if rank != 0:
        return None
    cpu = None
    if world == 1 and args.cpu_baseline_seconds > 0:
        ms, info = c3_cpu_sample(cfg, args.cpu_baseline_seconds, args.seed)
        cpu = dict(info, value=ms)
    return {
        "metric": "CABAttention layer ms @N=128k (dim 512, 8 heads)",
        "value": step_ms / world, "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (x iid N(0,1) bf16, seeded; weights N(0, 0.02^2) from the seed)",
        "config": {"workload": cfg["workload"], "per_rank": f"B={B} N={N} dim={dim} heads={H} head_dim={D}",
                   "parallelism": f"batch shards, {world} rank(s), no data-path collective",
                   "l2": "x 262 MB and qkv 786 MB per rank > 126 MB L2; no flush needed"},
        "stages": stages,
        "roofline": {"bound": "tensor", "kernel": "attn_tc_kernel<64> (block-sparse attention, head_dim 64)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} {peak_src}", "frac_of_sustained": achieved / tf_sus,
                     "traffic": ATTN_TRAFFIC_BYTES.get("c3")},
        "cpu_baseline": cpu,
        "e2e": {"value": te.item() / args.steps / world, "unit": "ms",
                "h2d_bytes_per_step": world * x_h.numel() * 2, "d2h_bytes_per_step": world * out_h.numel() * 2},
        # ours per forward: coarsen, two FRC GEMMs, top-k, pair-union, attention (the two
        # projections are cuBLAS GEMMs)
        "gpu_launches": 6 * args.steps,
        "clocks": clocks,
    }


def c3_cpu_sample(cfg, seconds_budget, seed=0):
    """The CABAttention layer on the host CPU: the predictor + attention sample of
    cpu_sample (head_dim 64) plus float32 torch projections of a row sample, extrapolated."""
    ms_pa, info = cpu_sample(cfg, seconds_budget * 0.8, seed)
    rows = 8192
    g = torch.Generator().manual_seed(seed)
    xs = torch.randn(rows, cfg["dim"], generator=g)
    w = torch.randn(4 * cfg["dim"], cfg["dim"], generator=g) * 0.02
    xs @ w.T
    t0 = time.perf_counter()
    xs @ w.T
    dt = time.perf_counter() - t0
    proj_ms = dt * 1e3 * cfg["B"] * cfg["N"] / rows
    info = dict(info, sample=info["sample"] + f"; projections: float32 torch GEMMs of {rows} rows "
                                                f"({dt:.3f} s), scaled to B*N rows", extrapolated=True)
    return ms_pa + proj_ms, info


# --------------------------------------------------------------------------- predictor sweep
def run_sweep_ours(args, cfg, rank, world, local_rank):
    """the predictor (coarsen -> FRC -> top-k) per N on device-resident q, k.
    Each N is timed over `steps` steps with CUDA events per stage; the line's value and
    roofline are those of the largest N, the others are in `sweep`."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    from cab_attention import CoarseCurvaturePredictor, _lib
    from cab_attention import roofline as rl
    from cab_attention.kernels import coarsen_qk_max_l2, compute_block_frc, topk_blocks
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    pred = CoarseCurvaturePredictor(block_size=BLOCK, sparsity=cfg["sparsity"], lambda_redundancy=LAMBDA)
    B, Hq, Hkv, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    sweep, last = {}, None
    for N in SWEEP_N:
        c = dict(cfg, N=N)
        q_h, k_h, _ = make_inputs(c, rank, args.seed, pin=True)
        q, k = q_h.to(dev), k_h.to(dev)
        kk = pred.keep_per_row(N)

        def step(ev=None):
            if ev: ev[0].record()
            qc, kc = coarsen_qk_max_l2(q, k, BLOCK)
            if ev: ev[1].record()
            frc, _, _ = compute_block_frc(qc, kc, 1.0, LAMBDA, return_affinity=False, return_redundancy=False)
            if ev: ev[2].record()
            idx, num, _ = topk_blocks(frc, kk, True, True, False, return_dense=False)
            if ev: ev[3].record()
            return idx, num

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        barrier()
        if N == SWEEP_N[-1]:
            sampler.mark_start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for st in range(args.steps):
            step(evs[st])
        end.record()
        barrier()
        if N == SWEEP_N[-1]:
            sampler.mark_end()
        t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        st_ms = [statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps))
                 for j in range(3)]
        # the same step captured in a CUDA graph: replays carry no per-call host work
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            graph.replay()
        g1.record()
        torch.cuda.synchronize()
        graph_ms = g0.elapsed_time(g1) / args.steps
        del graph
        M = (N + BLOCK - 1) // BLOCK
        sweep[str(N)] = {"ms": t.item() / args.steps, "graph_ms": graph_ms, "M": M, "k": kk,
                         "coarsen_ms": st_ms[0], "frc_ms": st_ms[1], "topk_ms": st_ms[2]}
        last = (N, M, kk, q_h, k_h, q, k, step, st_ms)
    clocks = sampler.stop()

    N, M, kk, q_h, k_h, q, k, step, st_ms = last
    # end to end at the largest N: pinned q, k in, block lists out, every step
    idx_h = torch.empty(B, Hq, M, kk, dtype=torch.int32).pin_memory()
    num_h = torch.empty(B, Hq, M, dtype=torch.int32).pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        qd, kd = q_h.to(dev, non_blocking=True), k_h.to(dev, non_blocking=True)
        idx, num = pred.predict_blocks(qd, kd)
        idx_h.copy_(idx, non_blocking=True)
        num_h.copy_(num, non_blocking=True)
    e1.record()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    c_ms, f_ms, k_ms = st_ms
    flop = rl.frc_flops(B, Hq, M, D)
    achieved = flop / f_ms / 1e9
    stages = {
        "coarsen": {"ms": c_ms, "GB/s": rl.coarsen_bytes(B, Hq, Hkv, N, D, 2, BLOCK) / c_ms / 1e6},
        "frc": {"ms": f_ms, "TFLOP/s": achieved},
        "topk": {"ms": k_ms, "GB/s": rl.topk_bytes(B, Hq, M, kk) / k_ms / 1e6},
    }
    if rank != 0:
        return None
    cpu = None
    if world == 1 and args.cpu_baseline_seconds > 0:
        ms, info = sweep_cpu_sample(dict(cfg, N=N), args.seed)
        cpu = dict(info, value=ms)
    return {
        "metric": "CAB predictor ms @N=128k (sweep over N)",
        "value": sweep[str(N)]["ms"] / world, "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sweep[str(N)]["ms"], "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K)",
        "config": {"workload": cfg["workload"], "per_rank": f"B={B} Hq={Hq} Hkv={Hkv} D={D}",
                   "parallelism": f"(batch x head) shards, {world} rank(s), no data-path collective",
                   "l2": "q, k at N=128k: 537 MB per rank > 126 MB L2; no flush needed"},
        "sweep": sweep,
        "stages": stages,
        "roofline": {"bound": "tensor", "kernel": "frc::gemm_kernel (A = Qc Kc^T, T = Direct Direct + F epilogue)",
                     "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s", "frac": achieved / tf_burst,
                     "peak_source": f"{peak_kind} bf16_tflops (burst: the GEMMs are timed alone)",
                     "traffic": None},
        "cpu_baseline": cpu,
        "e2e": {"value": te.item() / args.steps / world, "unit": "ms",
                "h2d_bytes_per_step": world * (q_h.numel() + k_h.numel()) * q_h.element_size(),
                "d2h_bytes_per_step": world * (idx_h.numel() + num_h.numel()) * 4},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }


def sweep_cpu_sample(cfg, seed=0):
    """The predictor (coarsen -> FRC -> top-k) of every head at N on the host CPU, float32
    torch on all threads (oracle/cab_torch_cpu.py)."""
    from oracle import cab_torch_cpu as tcpu
    from cab_attention import synthetic
    torch.set_num_threads(os.cpu_count())
    N, D = cfg["N"], cfg["D"]
    q, k, _ = synthetic.make_qkv(cfg["B"], cfg["Hq"], cfg["Hkv"], N, D, torch.bfloat16, seed)
    G = cfg["Hq"] // cfg["Hkv"]
    dt = 0.0
    for b in range(cfg["B"]):
        for h in range(cfg["Hq"]):
            qs, ks = q[b, h].float(), k[b, h // G].float()
            t0 = time.perf_counter()
            tcpu.predictor_head(qs, ks, BLOCK, cfg["sparsity"], LAMBDA)
            dt += time.perf_counter() - t0
    heads = cfg["B"] * cfg["Hq"]
    return dt * 1e3, {"unit": "ms", "cores": torch.get_num_threads(), "cpu_model": tcpu.cpu_model(),
                      "kind": "port", "dtype": "f32", "extrapolated": False, "measured_fraction": 1.0,
                      "sample": f"float32 torch predictor of all {heads} heads at N={N} ({dt:.2f} s)"}


def run_sweep_reference(args, cfg):
    """The reference path's CPU restatement of the predictor (oracle port) per N."""
    sweep, info = {}, {}
    for N in SWEEP_N:
        vals = []
        for _ in range(max(1, min(args.steps, 3))):
            ms, info = sweep_cpu_sample(dict(cfg, N=N), args.seed)
            vals.append(ms)
        sweep[str(N)] = {"ms": statistics.median(vals)}
    value = sweep[str(SWEEP_N[-1])]["ms"]
    return {
        "metric": "CAB predictor ms @N=128k (sweep over N)", "impl": "reference", "value": value,
        "unit": "ms", "n_gpus": 0, "steps": args.steps, "warmup": 0, "ms_per_step": value,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K)", "config": {"workload": cfg["workload"]},
        "sweep": sweep,
        "cpu_baseline": dict(info, value=value),
        "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- flash row
def flash_flop(cfg):
    from cab_attention import roofline as rl
    return rl.flash_attention_flops(cfg["B"], cfg["Hq"], cfg["N"], cfg["N"], cfg["D"])


def run_flash_ours(args, cfg, rank, world, local_rank):
    """Dense flash attention with cumulative scores through cab_flash_attn_fwd."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    from cab_attention.kernels.flash_attention_accumulate import flash_attention_forward
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    B, H, N, D = cfg["B"], cfg["Hq"], cfg["N"], cfg["D"]
    q_h, k_h, v_h = make_inputs(cfg, rank, args.seed, pin=True)
    q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    scores = torch.zeros(B, H, N, dtype=torch.float32, device=dev)
    out = torch.empty_like(q)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        scores.zero_()
        flash_attention_forward(q, k, v, scores=scores, out=out)
        flash_attention_forward(q, k, v, out=out)
    barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.2)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    barrier()
    sampler.mark_start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for st in range(args.steps):
        scores.zero_()
        flash_attention_forward(q, k, v, scores=scores, out=out)
    end.record()
    barrier()
    for st in range(args.steps):  # the same attention without the column scores
        ev[st][0].record()
        flash_attention_forward(q, k, v, out=out)
        ev[st][1].record()
    barrier()
    sampler.mark_end()
    clocks = sampler.stop()
    t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = t.item() / args.steps
    with_scores = start.elapsed_time(end) / args.steps  # includes the 1 MB score clear per step
    plain = statistics.mean(ev[s][0].elapsed_time(ev[s][1]) for s in range(args.steps))
    assert _flash_status() == 0
    # end to end: pinned host inputs in, output and scores out, every step
    out_h = torch.empty_like(q_h).pin_memory()
    sc_h = torch.empty(B, H, N, dtype=torch.float32).pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        qd, kd, vd = (x.to(dev, non_blocking=True) for x in (q_h, k_h, v_h))
        sd = torch.zeros(B, H, N, dtype=torch.float32, device=dev)
        od = flash_attention_forward(qd, kd, vd, scores=sd)
        out_h.copy_(od, non_blocking=True)
        sc_h.copy_(sd, non_blocking=True)
    e1.record()
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    flop = flash_flop(cfg)
    achieved = flop / with_scores / 1e9
    peak, peak_src = pick_peak(clocks, with_scores * args.steps, tf_burst, tf_sus)
    if rank != 0:
        return None
    cpu = None
    if world == 1 and args.cpu_baseline_seconds > 0:
        ms, desc = flash_cpu_sample(cfg, args.cpu_baseline_seconds, args.seed)
        cpu = {"value": ms, "unit": "ms", "cores": os.cpu_count(), "kind": "port", "sample": desc}
    return {
        "metric": "flash attention + cumulative scores ms @N=32k",
        "value": step_ms / world, "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K/V)",
        "config": {"workload": cfg["workload"], "per_rank": f"B={B} H={H} N={N} D={D}",
                   "l2": "inputs 201 MB per rank > 126 MB L2; no flush needed"},
        "stages": {"with_scores_ms": with_scores, "without_scores_ms": plain,
                   "scores_overhead": with_scores / plain - 1.0},
        "roofline": {"bound": "tensor", "kernel": "attn_tc_kernel<dense> (flash + column scores)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} {peak_src}", "traffic": None},
        "cpu_baseline": cpu,
        "e2e": {"value": te.item() / args.steps / world, "unit": "ms",
                "h2d_bytes_per_step": world * sum(x.numel() * x.element_size() for x in (q_h, k_h, v_h)),
                "d2h_bytes_per_step": world * (out_h.numel() * out_h.element_size() + sc_h.numel() * 4)},
        "gpu_launches": 2 * args.steps,  # workspace clear + attention kernel per step
        "clocks": clocks,
    }


def _flash_status():
    from cab_attention import _lib
    return _lib.device_status()


def flash_cpu_sample(cfg, seconds_budget, seed=0):
    """Oracle flash restatement on a bounded sample (query blocks of one head against all
    keys), extrapolated linearly to the whole workload."""
    from oracle import cab_oracle as orc
    from cab_attention import synthetic
    N, D = cfg["N"], cfg["D"]
    q = synthetic.normal_heads("q", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    k = synthetic.normal_heads("k", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    v = synthetic.normal_heads("v", [0], 1, N, D, torch.bfloat16, seed).float().numpy()
    nb, t = 1, 0.0
    while True:
        t0 = time.perf_counter()
        orc.flash_attention_cumulative(q[:, :, : 128 * nb], k, v)
        t = time.perf_counter() - t0
        if t * 2 > seconds_budget or 128 * nb * 2 > N:
            break
        nb *= 2
    blocks = cfg["B"] * cfg["Hq"] * ((N + 127) // 128)
    return t * 1e3 * blocks / nb, (f"numpy oracle: {nb} query blocks of 128 rows of one head against all "
                                   f"{N} keys ({t:.1f} s), extrapolated linearly to {blocks} blocks")


def run_flash_reference(args, cfg):
    """The reference's own Triton kernel (baseline/_ref) on this GPU when it is installed,
    else the oracle port on the host cores."""
    import importlib.util
    path = REPO / "baseline" / "_ref" / "cab_attention" / "kernels" / "flash_attention_accumulate.py"
    ref = None
    if path.exists() and torch.cuda.is_available():
        try:
            spec = importlib.util.spec_from_file_location("ref_flash_attention_accumulate", path)
            ref = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(ref)
        except Exception:
            ref = None
    base = {"metric": "flash attention + cumulative scores ms @N=32k", "impl": "reference", "unit": "ms",
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "data": "synthetic (iid N(0,1) per-(b,h) seeded Q/K/V)",
            "config": {"workload": cfg["workload"]}}
    if ref is None:
        ms, desc = flash_cpu_sample(cfg, args.reference_step_seconds, args.seed)
        base.update({"value": ms, "n_gpus": 0, "ms_per_step": ms, "dtype": "f64",
                     "cpu_baseline": {"value": ms, "unit": "ms", "cores": os.cpu_count(), "kind": "port",
                                      "sample": desc},
                     "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return base
    dev = torch.device("cuda", 0)
    q_h, k_h, v_h = make_inputs(cfg, 0, args.seed, pin=True)
    q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    for _ in range(args.warmup):
        ref.flash_attention_with_cumulative_scores(q, k, v)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ref.flash_attention_with_cumulative_scores(q, k, v)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    base.update({"value": ms, "n_gpus": 1, "ms_per_step": ms, "dtype": "bf16",
                 "kernel": "reference Triton kernel (baseline/_ref) on this GPU",
                 "cpu_baseline": None,
                 "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return base


# --------------------------------------------------------------------------- nodefrc / evict rows
def _aux_inputs(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    if cfg is CONFIGS["nodefrc"] or cfg.get("D") == 0:
        a = torch.rand(cfg["B"], cfg["N"], cfg["N"], generator=g)
        return a / a.sum(dim=-1, keepdim=True)
    return torch.rand(cfg["B"], cfg["N"], generator=g)


def _time_device(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_aux_ours(args, cfg, rank, world, local_rank):
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm, _, _, peak_kind = measured_peaks()
    x_h = _aux_inputs(cfg, args.seed + rank).pin_memory()
    x = x_h.to(dev)
    sampler = ClockSampler(local_rank)
    if args.config == "nodefrc":
        from cab_attention.kernels.frc_triton import compute_frc
        fn = lambda: compute_frc(x)  # noqa: E731
        metric = "node FRC ms (16 x 4096-node graphs)"
        nbytes = x.numel() * x.element_size()  # A crosses HBM once (second pass from L2)
        d2h = cfg["B"] * cfg["N"] * 4
        e2e_fn = lambda: compute_frc(x_h.to(dev, non_blocking=True)).cpu()  # noqa: E731
        launches = 2 * cfg["B"]
    else:
        from cab_attention.eviction import select_indices_batched
        K = cfg["D"]
        fn = lambda: select_indices_batched(cfg["N"], K, x, None, 0.3, 0.2)  # noqa: E731
        metric = "eviction selection ms (32 caches x 131072 tokens, keep 8192)"
        nbytes = x.numel() * 4
        d2h = cfg["B"] * (K * 8 + 16)

        def e2e_fn():
            keep, counts = select_indices_batched(cfg["N"], K, x_h.to(dev, non_blocking=True), None, 0.3, 0.2)
            return keep.cpu(), counts.cpu()
        launches = 2
    sampler.start()
    time.sleep(0.2)
    sampler.mark_start()
    ms = _time_device(fn, args.steps, args.warmup)
    sampler.mark_end()
    clocks = sampler.stop()
    e2e = _time_device(e2e_fn, args.steps, 1)
    achieved = nbytes / ms / 1e6
    return {
        "metric": metric, "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded torch.rand)", "config": {"workload": cfg["workload"]},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": None},
        "cpu_baseline": None,
        "e2e": {"value": e2e, "unit": "ms", "h2d_bytes_per_step": x.numel() * x.element_size(),
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches * args.steps, "clocks": clocks,
    }


def run_aux_reference(args, cfg):
    """The reference's own implementation (baseline/_ref) on this GPU: compute_frc (its
    default Triton path is O(N^3); compute_frc_pytorch, torch.matmul, is timed) and
    ThreeComponentEvictionPolicy.select_indices once per cache."""
    import importlib.util
    name = "kernels/frc_triton.py" if args.config == "nodefrc" else "eviction/policy.py"
    path = REPO / "baseline" / "_ref" / "cab_attention" / name
    base = {"metric": "node FRC ms (16 x 4096-node graphs)" if args.config == "nodefrc"
            else "eviction selection ms (32 caches x 131072 tokens, keep 8192)",
            "impl": "reference", "unit": "ms", "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "data": "synthetic (seeded torch.rand)", "config": {"workload": cfg["workload"]}}
    if not path.exists() or not torch.cuda.is_available():
        base["unavailable"] = "reference module or GPU missing"
        return base
    spec = importlib.util.spec_from_file_location("ref_aux", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    x = _aux_inputs(cfg, args.seed).cuda()
    if args.config == "nodefrc":
        fn = lambda: [ref.compute_frc_pytorch(x[b]) for b in range(x.shape[0])]  # noqa: E731
        kernel = "compute_frc_pytorch (torch.matmul) per graph on this GPU"
    else:
        pol = ref.ThreeComponentEvictionPolicy(ref.EvictionConfig(0.3, 0.2, 0.5))
        fn = lambda: [pol.select_indices(cfg["N"], cfg["D"], x[b], None, device="cuda")  # noqa: E731
                      for b in range(x.shape[0])]
        kernel = "ThreeComponentEvictionPolicy.select_indices per cache on this GPU"
    ms = _time_device(fn, args.steps, args.warmup)
    base.update({"value": ms, "n_gpus": 1, "ms_per_step": ms, "dtype": "f32", "kernel": kernel,
                 "cpu_baseline": None,
                 "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return base


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="ns")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-baseline-seconds", type=float, default=15.0)
    ap.add_argument("--reference-step-seconds", type=float, default=6.0)
    ap.add_argument("--no-flex", dest="flex", action="store_false",
                    help="skip the FlexAttention comparison on the same lists (1 GPU)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="--gpus N > 1: split one layer's (batch x head) units over the ranks and "
                         "all-gather the output (strong), or give every rank its own layer (weak)")
    ap.add_argument("--batch", type=int, default=None, help="override B per rank (profiling)")
    ap.add_argument("--heads", type=int, default=None,
                    help="override the KV-head count per rank, query heads scaled (profiling)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.batch is not None or args.heads is not None:
        G = cfg["Hq"] // cfg["Hkv"]
        cfg["B"] = args.batch if args.batch is not None else cfg["B"]
        cfg["Hkv"] = args.heads if args.heads is not None else cfg["Hkv"]
        cfg["Hq"] = cfg["Hkv"] * G
        cfg["workload"] += f" [reduced to B={cfg['B']} Hq={cfg['Hq']} Hkv={cfg['Hkv']}]"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            torch.set_num_threads(os.cpu_count())
            if args.config == "flash":
                res = run_flash_reference(args, cfg)
            elif args.config == "sweep":
                res = run_sweep_reference(args, cfg)
            elif args.config == "c3":
                res = run_reference(args, cfg, sampler=c3_cpu_sample,
                                    metric="CABAttention layer ms @N=128k (dim 512, 8 heads)")
            elif args.config in ("nodefrc", "evict"):
                res = run_aux_reference(args, cfg)
            else:
                res = run_reference(args, cfg)
            print(json.dumps(res), flush=True)
        return

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run = {"flash": run_flash_ours, "nodefrc": run_aux_ours, "evict": run_aux_ours,
               "sweep": run_sweep_ours, "c3": run_c3_ours}.get(args.config, run_ours)
        res = run(args, cfg, rank, world, local_rank)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
