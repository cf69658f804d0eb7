"""HuggingFace patch helpers of flash_attention_accumulate (no GPU needed for the patching
itself): which modules get patched, head counts taken from the config (Qwen2 style), and
where get_all_cumulative_scores finds the scores."""

import types

import torch

from cab_attention.kernels import flash_attention_accumulate as faa


class _Attn(torch.nn.Module):
    def __init__(self, heads=4, kv=2, d=8, with_counts=True, complete=True):
        super().__init__()
        self.head_dim = d
        self.q_proj = torch.nn.Linear(heads * d, heads * d, bias=False)
        self.k_proj = torch.nn.Linear(heads * d, kv * d, bias=False)
        self.v_proj = torch.nn.Linear(heads * d, kv * d, bias=False)
        if complete:
            self.o_proj = torch.nn.Linear(heads * d, heads * d, bias=False)
        if with_counts:
            self.num_heads, self.num_key_value_heads = heads, kv
        else:
            self.config = types.SimpleNamespace(num_attention_heads=heads, num_key_value_heads=kv)


def _model(attns):
    layers = torch.nn.ModuleList()
    for a in attns:
        layer = torch.nn.Module()
        layer.self_attn = a
        layers.append(layer)
    m = torch.nn.Module()
    m.model = torch.nn.Module()
    m.model.layers = layers
    return m


def test_patches_usable_modules_only(caplog):
    a0, a1, a2 = _Attn(), _Attn(with_counts=False), _Attn(complete=False)
    model = _model([a0, a1, a2])
    assert faa.replace_attention_with_flash(model) is model
    assert isinstance(a0.forward, faa._PatchedAttention)
    assert isinstance(a1.forward, faa._PatchedAttention)
    assert (a1.num_heads, a1.num_key_value_heads) == (4, 2)  # taken from the config
    assert not isinstance(a2.forward, faa._PatchedAttention)  # no o_proj
    assert "model.layers.2.self_attn" in caplog.text
    assert a0._flash_cumulative_scores is None


def test_module_filter_and_nothing_to_patch(caplog):
    a0, a1 = _Attn(), _Attn()
    faa.replace_attention_with_flash(_model([a0, a1]), module_filter=lambda name, m: name.endswith("1.self_attn"))
    assert not isinstance(a0.forward, faa._PatchedAttention)
    assert isinstance(a1.forward, faa._PatchedAttention)
    faa.replace_attention_with_flash(torch.nn.Linear(2, 2))
    assert "no decoder attention module" in caplog.text


def test_scores_from_patched_modules_then_wrappers():
    a0, a1 = _Attn(), _Attn()
    model = _model([a0, a1])
    faa.replace_attention_with_flash(model)
    assert faa.get_all_cumulative_scores(model) == {}
    a1._flash_cumulative_scores = torch.ones(1, 4, 3)
    got = faa.get_all_cumulative_scores(model)
    assert list(got) == ["model.layers.1.self_attn"]
    wrapped = torch.nn.Module()
    wrapped.att = faa.FlashAttentionWithAccumulation()
    wrapped.att.cumulative_scores = torch.zeros(1, 2, 5)
    assert list(faa.get_all_cumulative_scores(wrapped)) == ["att"]
