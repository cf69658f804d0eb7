"""Seeded synthetic inputs for the benchmark configurations and the parity tests.

The reference measures this path on synthetic tensors (``benchmarks/benchmark_predictor.py:73``,
``benchmarks/kernel_benchmark.py:76-77``: iid normal Q, K). Every (batch, head) slice is
drawn from its own generator seeded by (seed, b, h, tensor), so any shard of a larger
batch can be produced on its own and equals the same slice of the whole batch: sharded
runs need no broadcast.

Planted bridge (the acceptance case): key block j* of a KV head is overwritten with
1e-3 times the max-L2 token of query block i* (of one query head of that KV group), so the
coarse key of j* is exactly colinear with the coarse query of i* and tiny in magnitude:
a low-magnitude, structurally unique connection that the curvature score must keep.
"""

from __future__ import annotations

import torch

_TENSOR_IDS = {"q": 0, "k": 1, "v": 2, "x": 3}


def slice_generator(seed: int, b: int, h: int, name: str) -> torch.Generator:
    return torch.Generator().manual_seed(((seed * 1_000_003 + b) * 4099 + h) * 7 + _TENSOR_IDS[name])


def normal_heads(name: str, batches, heads: int, N: int, D: int, dtype: torch.dtype, seed: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``[len(batches), heads, N, D]`` iid N(0, 1) on the CPU; slice (b, h) is seeded by
    (seed, global batch index b, h, name)."""
    batches = list(batches)
    if out is None:
        out = torch.empty(len(batches), heads, N, D, dtype=dtype)
    for bi, b in enumerate(batches):
        for h in range(heads):
            g = slice_generator(seed, b, h, name)
            out[bi, h].copy_(torch.randn(N, D, generator=g, dtype=torch.float32))
    return out


def make_qkv(B: int, Hq: int, Hkv: int, N: int, D: int, dtype=torch.bfloat16, seed: int = 0,
             batch_offset: int = 0, pin: bool = False):
    """Q ``[B,Hq,N,D]``, K and V ``[B,Hkv,N,D]`` on the CPU (pinned when ``pin``)."""
    batches = range(batch_offset, batch_offset + B)

    def alloc(h):
        t = torch.empty(B, h, N, D, dtype=dtype)
        return t.pin_memory() if pin else t

    q = normal_heads("q", batches, Hq, N, D, dtype, seed, alloc(Hq))
    k = normal_heads("k", batches, Hkv, N, D, dtype, seed, alloc(Hkv))
    v = normal_heads("v", batches, Hkv, N, D, dtype, seed, alloc(Hkv))
    return q, k, v


def make_unit_qkv(units, G: int, N: int, D: int, dtype=torch.bfloat16, seed: int = 0, pin: bool = False):
    """Q ``[1, len(units)*G, N, D]``, K and V ``[1, len(units), N, D]`` holding the given
    ``(b, kv_head)`` units of a larger batch (query heads ``kv_head*G .. +G-1``), each slice
    drawn from its own seed: a rank's shard of the (batch x head) partition, equal to the
    same slices of ``make_qkv`` over the whole batch."""
    n = len(units)

    def alloc(h):
        t = torch.empty(1, h, N, D, dtype=dtype)
        return t.pin_memory() if pin else t

    q, k, v = alloc(n * G), alloc(n), alloc(n)
    for i, (b, g) in enumerate(units):
        for j in range(G):
            q[0, i * G + j].copy_(torch.randn(N, D, generator=slice_generator(seed, b, g * G + j, "q")))
        k[0, i].copy_(torch.randn(N, D, generator=slice_generator(seed, b, g, "k")))
        v[0, i].copy_(torch.randn(N, D, generator=slice_generator(seed, b, g, "v")))
    return q, k, v


def max_l2_token(x_block: torch.Tensor) -> torch.Tensor:
    """Row of ``x_block [n, D]`` with the largest L2 norm (fp64 norms, first max wins)."""
    n = (x_block.double() ** 2).sum(-1)
    return x_block[int(torch.argmax(n))]


def bridge_positions(M: int, count: int, seed: int, causal: bool = False):
    """``count`` distinct (i*, j*) block pairs with i* != j* (j* < i* when causal)."""
    g = torch.Generator().manual_seed(seed * 7919 + 17)
    out = []
    while len(out) < count:
        i, j = (int(x) for x in torch.randint(0, M, (2,), generator=g))
        if i == j or (causal and j > i) or (i, j) in out:
            continue
        out.append((i, j))
    return out


def plant_bridge(q: torch.Tensor, k: torch.Tensor, b: int, hq: int, i_star: int, j_star: int,
                 block_size: int = 64, scale: float = 1e-3) -> None:
    """In place: every token of key block j* of KV head hq // (Hq // Hkv) in batch b
    becomes ``scale`` * (max-L2 token of query block i* of query head hq)."""
    G = q.shape[1] // k.shape[1]
    N = q.shape[2]
    qi = q[b, hq, i_star * block_size:min(N, (i_star + 1) * block_size)]
    rep = (max_l2_token(qi).float() * scale).to(k.dtype)
    j0, j1 = j_star * block_size, min(N, (j_star + 1) * block_size)
    k[b, hq // G, j0:j1] = rep


def make_config(name: str, seed: int = 0, batch_offset: int = 0, batches: int | None = None,
                pin: bool = False):
    """Inputs of a named configuration. Returns a dict with q, k, v (CPU), the predictor
    settings and the planted bridges [(b, hq, i*, j*)]."""
    cfgs = {
        # CPU-oracle case
        "c1": dict(B=1, Hq=8, Hkv=8, N=4096, D=64, dtype=torch.float32, sparsity=0.90,
                   causal=False, bridges=0),
        # bf16 predictor + attention with one planted bridge per (b, h)
        "c2": dict(B=2, Hq=8, Hkv=8, N=32768, D=128, dtype=torch.bfloat16, sparsity=0.95,
                   causal=False, bridges=1),
        # north_star shape: B2 H8 N128000 D128, s=0.95
        "ns": dict(B=2, Hq=8, Hkv=8, N=128000, D=128, dtype=torch.bfloat16, sparsity=0.95,
                   causal=False, bridges=0),
        # GQA 32/8, causal, s=0.99, 4 planted bridges
        "c5": dict(B=1, Hq=32, Hkv=8, N=65536, D=128, dtype=torch.bfloat16, sparsity=0.99,
                   causal=True, bridges=4),
    }
    c = dict(cfgs[name])
    B = c["B"] if batches is None else batches
    q, k, v = make_qkv(B, c["Hq"], c["Hkv"], c["N"], c["D"], c["dtype"], seed, batch_offset, pin)
    M = (c["N"] + 63) // 64
    planted = []
    if c["bridges"] and name == "c2":
        for bi in range(B):
            for h in range(c["Hq"]):
                (i, j), = bridge_positions(M, 1, seed * 1000 + (batch_offset + bi) * 64 + h)
                plant_bridge(q, k, bi, h, i, j)
                planted.append((bi, h, i, j))
    elif c["bridges"] and name == "c5":
        g = torch.Generator().manual_seed(seed * 31 + 5)
        heads = torch.randperm(c["Hkv"], generator=g)[: c["bridges"]].tolist()
        pos = bridge_positions(M, c["bridges"], seed + 101, causal=True)
        for (kvh, (i, j)) in zip(heads, pos):
            hq = kvh * (c["Hq"] // c["Hkv"])
            for bi in range(B):
                plant_bridge(q, k, bi, hq, i, j)
                planted.append((bi, hq, i, j))
    c.update(q=q, k=k, v=v, bridges_planted=planted, M=M, lambda_redundancy=0.5, block_size=64)
    return c
