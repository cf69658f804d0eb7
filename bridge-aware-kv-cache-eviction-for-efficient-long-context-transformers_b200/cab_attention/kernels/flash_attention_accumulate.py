"""Flash attention with cumulative column scores (``cab_attention/kernels/
flash_attention_accumulate.py`` of the reference), on the sm_100a kernel ``cab_flash_attn_fwd``.

``flash_attention_with_cumulative_scores(q, k, v, cumulative_scores=None, scale=None)``
returns ``(output, cumulative_scores)`` exactly as the reference's wrapper
(``flash_attention_accumulate.py:169-261``): ``output = softmax(q k^T * scale) v``
(non-causal) and ``cumulative_scores [B, H, N_k] += sum_i exp(s_ij - m_i(j))``, where
``m_i(j)`` is query i's running maximum over the 128-key blocks up to and including key
j's block (the reference kernel accumulates ``tl.sum(p, axis=0)`` with the running max of
each block, ``:117-156``). An existing ``cumulative_scores`` shorter than ``N_k`` is
extended with zeros first (``:223-230``), so scores keep accumulating across decode steps.

The HF integration helpers (``replace_attention_with_flash``, ``get_all_cumulative_scores``,
``FlashAttentionWithAccumulation``) keep the reference module's interface (``:264-598``:
names, signatures, the module attribute holding the scores, the layer-name keys);
``apply_rotary_pos_emb``, ``rotate_half`` and ``repeat_kv`` are HuggingFace's standard
functions. Grouped-query attention runs natively (each query head reads KV head
``h // (Hq // Hkv)``), which gives the same result as expanding K/V with ``repeat_kv`` first.
"""

from __future__ import annotations

import logging
import math
from typing import Optional, Tuple

import torch

from .. import _lib

logger = logging.getLogger(__name__)


def _prep(t: torch.Tensor) -> torch.Tensor:
    if t.stride(3) != 1 or any((s * t.element_size()) % 16 for s in t.stride()[:3]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def flash_attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            scores: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                            causal: bool = False, out: Optional[torch.Tensor] = None,
                            return_lse: bool = False):
    """Dense attention on ``cab_flash_attn_fwd``. ``q [B,Hq,Nq,D]``, ``k, v [B,Hkv,Nk,D]``
    (bf16/f16, D in {64, 128}); ``scores`` (fp32 ``[B,Hq,Nk]``, contiguous) is accumulated
    into when given. Returns ``out`` (and the natural-log LSE ``[B,Hq,Nq]``)."""
    _lib.require_cuda(q, k, v, scores)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape:
        raise ValueError("q must be [B, Hq, Nq, D] and k, v [B, Hkv, Nk, D]")
    B, Hq, Nq, D = q.shape
    Hkv, Nk = k.shape[1], k.shape[2]
    if k.shape[0] != B or k.shape[3] != D or Hq % Hkv:
        raise ValueError("k and v must be [B, Hkv, Nk, D] with Hq % Hkv == 0")
    if scores is not None:
        if scores.dtype != torch.float32 or tuple(scores.shape) != (B, Hq, Nk) or not scores.is_contiguous():
            raise ValueError(f"scores must be a contiguous float32 tensor [B, Hq, Nk] = {(B, Hq, Nk)}")
    q, k, v = _prep(q), _prep(k), _prep(v)
    if out is None:
        out = torch.empty(B, Hq, Nq, D, dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, Hq, Nq, D) or out.dtype != q.dtype or out.stride(3) != 1:
        raise ValueError("out must be [B, Hq, Nq, D] of q's dtype with a dense last dimension")
    lse = torch.empty(B, Hq, Nq, dtype=torch.float32, device=q.device) if return_lse else None
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    dt = _lib.dtype_code(q)
    L = _lib.lib()
    nbytes = _lib._c_size(0)
    _lib.check(L.cab_flash_attn_workspace_size(B, Hq, Nq, Nk, D, dt, int(scores is not None), nbytes),
               "cab_flash_attn_workspace_size")
    ws = _lib.workspace(nbytes.value, q.device)
    rc = L.cab_flash_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _lib.ptr(scores),
                              _lib.ptr(lse), B, Hq, Hkv, Nq, Nk, D, _lib.strides3(q), _lib.strides3(k),
                              _lib.strides3(v), _lib.strides3(out), sc, int(bool(causal)), dt,
                              _lib.ptr(ws), nbytes.value, _lib.stream_of(q))
    _lib.check(rc, "cab_flash_attn_fwd")
    return (out, lse) if return_lse else out


def flash_attention_with_cumulative_scores(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                           cumulative_scores: Optional[torch.Tensor] = None,
                                           scale: Optional[float] = None
                                           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(output [B,H,N_q,D], cumulative_scores [B,H,N_k])``; see the module docstring.
    Supports self-attention (``N_q == N_k``) and KV-cache steps (``N_q < N_k``)."""
    B, H, N_q, D = q.shape
    N_k = k.shape[2]
    if cumulative_scores is None:
        cumulative_scores = torch.zeros(B, H, N_k, dtype=torch.float32, device=q.device)
    elif cumulative_scores.shape[2] < N_k:
        ext = torch.zeros(B, H, N_k - cumulative_scores.shape[2], dtype=torch.float32, device=q.device)
        cumulative_scores = torch.cat([cumulative_scores, ext], dim=2)
    if cumulative_scores.dtype != torch.float32 or not cumulative_scores.is_contiguous():
        cumulative_scores = cumulative_scores.float().contiguous()
    output = flash_attention_forward(q, k, v, scores=cumulative_scores, scale=scale)
    return output, cumulative_scores


class FlashAttentionWithAccumulation(torch.nn.Module):
    """Attention module that keeps the cumulative column scores across calls
    (``flash_attention_accumulate.py:264-371``)."""

    def __init__(self, original_attention: Optional[torch.nn.Module] = None, accumulate_scores: bool = True):
        super().__init__()
        self.original_attention = original_attention
        self.accumulate_scores = accumulate_scores
        self.cumulative_scores = None
        self.reset_scores()

    def reset_scores(self):
        """Reset the cumulative scores (start of a new sequence)."""
        self.cumulative_scores = None

    def get_cumulative_scores(self) -> Optional[torch.Tensor]:
        return self.cumulative_scores

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, **kwargs):
        """``[B, H, N, D]`` inputs (or ``[B, N, H, D]``, detected as in the reference) ->
        ``(output, None)``."""
        transpose_back = query.dim() == 4 and query.shape[1] != key.shape[1]
        if transpose_back:
            query, key, value = (t.transpose(1, 2) for t in (query, key, value))
        if self.accumulate_scores:
            output, self.cumulative_scores = flash_attention_with_cumulative_scores(
                query, key, value, self.cumulative_scores)
        else:
            output = flash_attention_forward(query, key, value)
        if transpose_back:
            output = output.transpose(1, 2).contiguous()
        return output, None


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Rotates half the hidden dims of the input (RoPE)."""
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """RoPE with cos/sin ``[B, L, D]`` (HuggingFace layout)."""
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
    """``[B, Hkv, L, D] -> [B, Hkv * n_rep, L, D]`` (each KV head repeated n_rep times)."""
    batch, num_key_value_heads, slen, head_dim = hidden_states.shape
    if n_rep == 1:
        return hidden_states
    hidden_states = hidden_states[:, :, None, :, :].expand(batch, num_key_value_heads, n_rep, slen, head_dim)
    return hidden_states.reshape(batch, num_key_value_heads * n_rep, slen, head_dim)


# ---------------------------------------------------------------- HuggingFace integration
# Interface kept from the reference (flash_attention_accumulate.py:370-598): patched modules
# keep their running scores in the attribute ``_flash_cumulative_scores``, and the scores
# dictionary is keyed "model.layers.<i>.self_attn". The code below is this package's own.

_SCORES_ATTR = "_flash_cumulative_scores"
_PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj")


def _decoder_attention(model: torch.nn.Module):
    """Yields ``(name, layer index, module)`` for each ``model.model.layers[i].self_attn``."""
    layers = getattr(getattr(model, "model", None), "layers", None)
    for i, layer in enumerate(layers if layers is not None else ()):
        attn = getattr(layer, "self_attn", None)
        if attn is not None:
            yield f"model.layers.{i}.self_attn", i, attn


def _head_counts(attn: torch.nn.Module):
    """(query heads, KV heads) of an attention module, read from the module itself or,
    for modules that only carry them in their config (Qwen2 style), from ``attn.config``
    (then also set on the module); None when neither has them."""
    cfg = getattr(attn, "config", None)
    found = []
    for own, from_cfg in (("num_heads", "num_attention_heads"), ("num_key_value_heads", "num_key_value_heads")):
        n = getattr(attn, own, None)
        if n is None:
            n = getattr(cfg, from_cfg, None)
        if n is None:
            return None
        found.append(int(n))
    attn.num_heads, attn.num_key_value_heads = found
    return tuple(found)


class _PatchedAttention:
    """Replacement ``forward`` of a HuggingFace decoder attention module (Qwen2 / Llama
    call signature): the module's own projections and rotary embedding, its KV-cache
    update, then attention with cumulative column scores; the running scores live on the
    module. Returns ``(output, None)``: no attention weights are materialised."""

    def __init__(self, module: torch.nn.Module, layer_idx: int):
        self.module = module
        self.layer_idx = layer_idx
        if not hasattr(module, _SCORES_ATTR):
            setattr(module, _SCORES_ATTR, None)

    def _heads(self, proj: torch.nn.Module, x: torch.Tensor, n: int) -> torch.Tensor:
        b, t, _ = x.shape
        return proj(x).view(b, t, n, self.module.head_dim).transpose(1, 2)

    def __call__(self, hidden_states: torch.Tensor, position_embeddings: tuple,
                 attention_mask: Optional[torch.Tensor] = None, past_key_values=None,
                 cache_position: Optional[torch.LongTensor] = None, **kwargs):
        m = self.module
        cos, sin = position_embeddings
        q = self._heads(m.q_proj, hidden_states, m.num_heads)
        k = self._heads(m.k_proj, hidden_states, m.num_key_value_heads)
        v = self._heads(m.v_proj, hidden_states, m.num_key_value_heads)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx,
                                          cache_kwargs={"sin": sin, "cos": cos, "cache_position": cache_position})
        # KV heads are shared by their query-head group inside the kernel (no repeat_kv copy)
        ctx, scores = flash_attention_with_cumulative_scores(q, k, v, getattr(m, _SCORES_ATTR))
        setattr(m, _SCORES_ATTR, scores)
        b, _, t, _ = ctx.shape
        return m.o_proj(ctx.transpose(1, 2).reshape(b, t, -1)), None


def replace_attention_with_flash(model: torch.nn.Module, module_filter=None) -> torch.nn.Module:
    """Routes the attention of every decoder layer (``model.model.layers[i].self_attn``
    with q/k/v/o projections, a ``head_dim`` and known head counts) through this
    package's kernel, in place; ``module_filter(name, module)`` may exclude modules.
    Returns the model."""
    done, skipped = [], []
    for name, i, attn in _decoder_attention(model):
        if module_filter is not None and not module_filter(name, attn):
            continue
        usable = all(hasattr(attn, a) for a in _PROJECTIONS + ("head_dim",)) and _head_counts(attn) is not None
        if not usable:
            skipped.append(name)
            continue
        attn.forward = _PatchedAttention(attn, i)
        done.append(name)
    for name in skipped:
        logger.warning("%s left unpatched: no q/k/v/o projections, head_dim or head counts", name)
    if done:
        logger.info("flash attention with cumulative scores in %d module(s)", len(done))
    else:
        logger.warning("replace_attention_with_flash found no decoder attention module to patch")
    return model


def get_all_cumulative_scores(model: torch.nn.Module) -> dict:
    """``{module name: cumulative scores [B, H, N]}``: from the modules patched by
    ``replace_attention_with_flash`` or, if there are none, from
    ``FlashAttentionWithAccumulation`` wrappers anywhere in the model."""
    patched = {name: getattr(attn, _SCORES_ATTR) for name, _, attn in _decoder_attention(model)
               if getattr(attn, _SCORES_ATTR, None) is not None}
    if patched:
        return patched
    return {name: mod.get_cumulative_scores() for name, mod in model.named_modules()
            if isinstance(mod, FlashAttentionWithAccumulation) and mod.get_cumulative_scores() is not None}
