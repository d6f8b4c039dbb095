"""The training hook's host logic on the CPU (no kernel runs): the per-forward geometry (real indices under padding and
packed documents, prefill columns) must give the reference's masks exactly (the reference's train.py _Layout, from
the staged copy under oracle/_ref), for both rules and both layer kinds; and the hook's plumbing on a small model with
the LFM3 module structure: stock mode equals the unpatched model, remove() restores it, and the refusals of the
reference (double patch, unknown mode / rule, past_key_values, non-2D masks) hold."""
import importlib.util
import os

import pytest
import torch

import _lfm3_stub as stub
from lfm3_kv800 import train as T

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TRAIN = os.path.join(ROOT, "oracle", "_ref", "lfm3_kv800", "train.py")


@pytest.fixture(scope="module")
def ref_train():
    if not os.path.exists(REF_TRAIN):
        pytest.skip("the reference package is not staged under oracle/_ref (oracle/stage_reference.py)")
    spec = importlib.util.spec_from_file_location("ref_lfm3_train", REF_TRAIN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _same_masks(ref_train, B, Tn, rule, **kw):
    ours = T._Geometry(B, Tn, "cpu", rule, **kw)
    ref = ref_train._Layout(B, Tn, "cpu", rule, **kw)
    for kind in ("quant", "win"):
        a, b = ours.mask(kind), ref.mask(kind)
        assert a.shape == b.shape and torch.equal(a, b), (rule, kind, kw.keys())
    return ours


@pytest.mark.parametrize("rule", T.RULES)
@pytest.mark.parametrize("Tn", [1, 255, 384, 700, 1100])
def test_plain_masks_match_reference(ref_train, rule, Tn):
    g = _same_masks(ref_train, 2, Tn, rule)
    assert g.plain


@pytest.mark.parametrize("rule", T.RULES)
def test_padded_packed_prefill_masks_match_reference(ref_train, rule):
    B, Tn = 3, 900
    am = torch.ones(B, Tn, dtype=torch.long)
    am[1, :37] = 0                       # left padding
    am[2, 650:] = 0                      # right padding
    _same_masks(ref_train, B, Tn, rule, attention_mask=am)
    pos = torch.cat((torch.arange(400), torch.arange(300), torch.arange(200)))[None].expand(B, Tn)
    _same_masks(ref_train, B, Tn, rule, position_ids=pos)                          # packed documents
    _same_masks(ref_train, B, Tn, rule, attention_mask=am, position_ids=pos)
    _same_masks(ref_train, B, Tn, rule, prefill=512)                               # one prefill boundary
    _same_masks(ref_train, B, Tn, rule, attention_mask=am, prefill=torch.tensor([384, 700, 0]))
    g = _same_masks(ref_train, B, Tn, rule, attention_mask=am, position_ids=pos, prefill=300)
    assert not g.plain


def test_compaction_layout_matches_reference(ref_train):
    """The compact buffer for the K groups: documents at 256-aligned offsets, pads sent to the dump row."""
    B, Tn = 2, 800
    am = torch.ones(B, Tn, dtype=torch.long)
    am[1, :100] = 0
    pos = torch.cat((torch.arange(500), torch.arange(300)))[None].expand(B, Tn)
    ours = T._Geometry(B, Tn, "cpu", "cache", attention_mask=am, position_ids=pos)
    ref = ref_train._Layout(B, Tn, "cpu", "cache", attention_mask=am, position_ids=pos)
    assert ours.Tc == ref.Tc
    assert torch.equal(ours.to_compact, ref.comp_scatter) and torch.equal(ours.from_compact, ref.comp_gather)
    assert torch.equal(ours.r, ref.r) and torch.equal(ours.complete, ref.complete)


def test_stock_mode_and_remove_restore_the_model():
    m = stub.make_model(1)
    x = torch.randint(0, 97, (2, 300))
    ref = m(x).logits
    hook = T.patch_for_training(m, mode="stock")
    try:
        assert torch.equal(m(x).logits, ref)
        for l in T.QUANT_LAYERS + T.WINDOW_LAYERS:
            assert "forward" in m.model.layers[l].self_attn.__dict__
    finally:
        hook.remove()
    for l in T.QUANT_LAYERS + T.WINDOW_LAYERS:
        assert "forward" not in m.model.layers[l].self_attn.__dict__
    assert torch.equal(m(x).logits, ref)
    hook.remove()                         # idempotent


def test_hook_refusals():
    m = stub.make_model(2)
    with pytest.raises(ValueError):
        T.patch_for_training(m, rule="everything")
    hook = T.patch_for_training(m)
    try:
        with pytest.raises(RuntimeError):
            T.patch_for_training(m)       # already patched
        with pytest.raises(ValueError):
            hook.set_mode("fp8")
        x = torch.randint(0, 97, (1, 64))
        with pytest.raises(RuntimeError):
            m.model(x, past_key_values=object())
        with pytest.raises(RuntimeError):
            m.model(x, attention_mask=torch.ones(1, 1, 64, 64))
        with hook.using("stock"):
            assert hook.mode == "stock"
        assert hook.mode == "800h"
        with hook.prefill(32):
            assert hook._prefill == 32
        assert hook._prefill is None
    finally:
        hook.remove()
    bad = stub.make_model(3)
    bad.config.layer_types[6] = "conv"
    bad.model.config.layer_types[6] = "conv"
    with pytest.raises(ValueError):
        T.patch_for_training(bad)


def test_fp32_rope_rebuilt_and_restored():
    m = stub.make_model(4)
    m.model.rotary_emb = stub.Rotary(m.config, dtype=torch.bfloat16)
    low = m.model.rotary_emb
    hook = T.patch_for_training(m, mode="stock")
    assert m.model.rotary_emb is not low and m.model.rotary_emb.inv_freq.dtype == torch.float32
    hook.remove()
    assert m.model.rotary_emb is low
