"""float32 PyTorch restatement of the CAB prefill path on the host CPU -- TEST AND
MEASUREMENT INFRASTRUCTURE ONLY (the CPU baseline).

Like ``cab_oracle.py`` this is never imported by the product package. It is used by
``bench.py``'s ``cpu_baseline`` and ``--impl reference`` legs (the timed CPU baseline of
the reference's path) and by ``tests/test_cpu_baseline.py``, which checks it against the
float64 numpy oracle.

It computes the same stages with the same semantics as ``cab_oracle.py`` (which cites the
reference's call sites for each), in float32 torch with batched kernels on all host
threads, the way the reference's own PyTorch path runs on a CPU:

* coarsening: per 64-token block the token with the largest L2 norm
  (``coarsen_qk_max_l2_pytorch``; ``CAB_Attention_Colab.ipynb`` cells 5/7), norms in
  float32 here;
* FRC: ``A = Qc Kc^T / sqrt(D)``, Direct ``|A|``, ``T = Direct Direct``,
  ``F = Direct - lambda T`` (``benchmarks/kernel_benchmark.py:135-149``; torch.matmul as
  there);
* mask: per row the diagonal plus the top k-1 other blocks by F (``torch.topk``, as the
  reference's ``generate_block_mask`` callers, ``methods.py:339-345``);
* attention: softmax over the kept blocks' keys, fully masked rows -> 0
  (``methods.py:103-119,348-356``). The reference's manual path materialises a token mask of
  N x N per head (16 GB per head at N = 128000, not runnable); here the kept K / V blocks of
  a chunk of query blocks are gathered and multiplied with ``bmm``, which is the same
  arithmetic without the masked-out products.
"""

from __future__ import annotations

import math
import time

import torch


def coarsen(x: torch.Tensor, block: int):
    """``x [N, D]`` float32 -> (``x_coarse [M, D]``, ``idx [M]``), one token per block."""
    N, D = x.shape
    M = (N + block - 1) // block
    pad = M * block - N
    nrm = (x * x).sum(-1)
    if pad:
        nrm = torch.cat([nrm, torch.full((pad,), -math.inf)])
    local = nrm.view(M, block).argmax(-1)
    idx = torch.arange(M) * block + local
    return x[idx], idx


def predictor_head(q: torch.Tensor, k: torch.Tensor, block: int = 64, sparsity: float = 0.95,
                   lam: float = 0.5):
    """Coarsen -> FRC -> top-k for one head (non-causal, diagonal kept, highest F):
    ``q, k [N, D]`` float32 -> ``kv_idx [M, k]`` ascending (int64) and ``kv_num [M]``."""
    qc, _ = coarsen(q, block)
    kc, _ = coarsen(k, block)
    M, D = qc.shape
    direct = (qc @ kc.T).mul_(1.0 / math.sqrt(D)).abs_()
    frc = direct - lam * (direct @ direct)
    kk = max(1, int(M * (1.0 - sparsity)))
    frc.diagonal().fill_(math.inf)  # keep_diagonal: block i first, then the top k-1 others
    kv_idx = frc.topk(kk, dim=-1).indices.sort(dim=-1).values
    return kv_idx, torch.full((M,), kk, dtype=torch.int64)


def attention_head(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_idx: torch.Tensor,
                   block: int = 64, qblocks=None, chunk: int = 32) -> torch.Tensor:
    """Non-causal block-sparse attention of one head over its kept blocks (every row keeps
    the same count, as the non-causal top-k gives). ``qblocks`` restricts the work to
    those query blocks (timing samples); other rows stay 0."""
    N, D = q.shape
    M = (N + block - 1) // block
    pad = M * block - N
    if pad:
        z = torch.zeros(pad, D)
        q, k, v = torch.cat([q, z]), torch.cat([k, z]), torch.cat([v, z])
    qb = q.view(M, block, D)
    kf, vf = k.view(M, block * D), v.view(M, block * D)  # one row per key block
    keyvalid = (torch.arange(M * block) < N).view(M, block)
    out = torch.zeros(M, block, D)
    blocks = torch.arange(M) if qblocks is None else torch.as_tensor(qblocks)
    scale = 1.0 / math.sqrt(D)
    kk = kv_idx.shape[1]
    # gathered K / V of a chunk of query blocks (index_select into preallocated buffers:
    # advanced indexing of the block view is two orders of magnitude slower on the CPU)
    kbuf = torch.empty(chunk * kk, block * D)
    vbuf = torch.empty(chunk * kk, block * D)
    for c0 in range(0, len(blocks), chunk):
        bi = blocks[c0:c0 + chunk]
        n = len(bi)
        sel = kv_idx[bi].flatten()
        ks = torch.index_select(kf, 0, sel, out=kbuf[:n * kk]).view(n, kk * block, D)
        vs = torch.index_select(vf, 0, sel, out=vbuf[:n * kk]).view(n, kk * block, D)
        s = torch.bmm(qb[bi], ks.transpose(1, 2)).mul_(scale)
        if pad:
            s.masked_fill_(~keyvalid[kv_idx[bi]].flatten(1, 2)[:, None, :], -math.inf)
        p = torch.softmax(s, dim=-1)
        out[bi] = torch.bmm(p, vs)
    return out.view(M * block, D)[:N]


def layer_timed(q, k, v, block=64, sparsity=0.95, lam=0.5, budget_s=15.0):
    """Time the layer on ``q [B, Hq, N, D]``, ``k, v [B, Hkv, N, D]`` (any float dtype,
    converted per head to float32): whole heads (predictor, then attention over its kept
    blocks) until ``budget_s`` is spent (at least one), extrapolated linearly to every head
    (each head is the same work). Returns (ms per layer, dict of details)."""
    B, Hq, N, D = q.shape
    G = Hq // k.shape[1]
    heads = [(b, h) for b in range(B) for h in range(Hq)]
    t_pred = t_att = 0.0
    done = 0
    for (b, h) in heads:
        qs, ks, vs = q[b, h].float(), k[b, h // G].float(), v[b, h // G].float()
        t0 = time.perf_counter()
        kv_idx, _ = predictor_head(qs, ks, block, sparsity, lam)
        t1 = time.perf_counter()
        attention_head(qs, ks, vs, kv_idx, block)
        t2 = time.perf_counter()
        t_pred += t1 - t0
        t_att += t2 - t1
        done += 1
        if t_pred + t_att > budget_s:
            break
    scale = len(heads) / done
    info = {"predictor_ms": t_pred * 1e3 * scale, "attention_ms": t_att * 1e3 * scale,
            "heads_measured": done, "heads": len(heads), "measured_fraction": done / len(heads),
            "extrapolated": done < len(heads)}
    return (t_pred + t_att) * 1e3 * scale, info


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
