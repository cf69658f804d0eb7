"""The reference's GPU attention step, FlexAttention, fed the same kept-block lists --
TEST AND MEASUREMENT INFRASTRUCTURE ONLY (a same-box bar and an independent second check of
the block-sparse attention kernel; never imported by the product package).

The reference runs its block-sparse attention "with FlexAttention or manual sparse
attention" (``README.md:44-46``; ``requirements.txt:4-5``: torch >= 2.1, 2.5+ recommended for
FlexAttention). Here ``torch.nn.attention.flex_attention`` of the installed torch is given a
``BlockMask`` built with ``BlockMask.from_kv_blocks`` from this library's ``kv_idx`` /
``kv_num`` at ``BLOCK_SIZE = 64`` (the predictor's block size):

* every kept (query block, key block) pair is passed as a *full* block, so the compiled
  kernel evaluates no per-element mask inside it and skips every other block;
* the ``mask_mod`` looks the pair up in the dense block mask, which defines the same
  attention for any path that evaluates it (the eager implementation does);
* for causal masks the diagonal blocks are passed as partial blocks and the ``mask_mod``
  adds ``kv <= q``.

``from_kv_blocks`` takes the KV length from the index tensor's last dimension, so the lists
are padded to ``[B, H, M, M]``. The compiled kernel's tiles must divide the block size, so it
runs with ``BLOCK_M = BLOCK_N = 64`` (its default BLOCK_M of 128 is rejected for 64-token
blocks).
"""

from __future__ import annotations

import torch


def block_mask(kv_idx: torch.Tensor, kv_num: torch.Tensor, N: int, block: int = 64, causal: bool = False):
    """BlockMask of the kept blocks ``kv_idx [B, H, M, k]`` (ascending, first ``kv_num``
    valid) for a sequence of N tokens."""
    from torch.nn.attention.flex_attention import BlockMask

    B, H, M, k = kv_idx.shape
    dev = kv_idx.device
    valid = torch.arange(k, device=dev)[None, None, None, :] < kv_num[..., None]
    # padding entries go to a spare column M, dropped after the scatter
    dense = torch.zeros(B, H, M, M + 1, dtype=torch.bool, device=dev)
    dense.scatter_(3, torch.where(valid, kv_idx, M).long(), True)
    dense = dense[..., :M].contiguous()
    diag = torch.zeros_like(dense)
    if causal:
        diag = dense & torch.eye(M, dtype=torch.bool, device=dev)
    full = dense & ~diag

    def lists(mask):
        num = mask.sum(-1, dtype=torch.int32)
        # indices of the set blocks first, in ascending order, then padding
        order = torch.argsort((~mask).to(torch.int8), dim=-1, stable=True).to(torch.int32)
        return num, order

    full_num, full_idx = lists(full)
    part_num, part_idx = lists(diag)

    def mask_mod(b, h, q_idx, kv):
        keep = dense[b, h, q_idx // block, kv // block]
        if causal:
            keep = keep & (kv <= q_idx)
        return keep

    return BlockMask.from_kv_blocks(part_num, part_idx, full_num, full_idx, BLOCK_SIZE=block,
                                    mask_mod=mask_mod, seq_lengths=(N, N))


_compiled = None


def attention(q, k, v, bmask, scale=None):
    """Compiled ``flex_attention`` (GQA through ``enable_gqa`` when Hq != Hkv)."""
    global _compiled
    from torch.nn.attention.flex_attention import flex_attention

    if _compiled is None:
        _compiled = torch.compile(flex_attention, dynamic=False)
    gqa = q.shape[1] != k.shape[1]
    # the compiled kernel's tiles must divide the 64-token blocks (its default BLOCK_M is 128)
    bs = bmask.BLOCK_SIZE
    return _compiled(q, k, v, block_mask=bmask, scale=scale, enable_gqa=gqa,
                     kernel_options={"BLOCK_M": bs[0], "BLOCK_N": bs[1]})
