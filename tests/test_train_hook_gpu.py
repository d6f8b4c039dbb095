"""The training hook on the GPU, against the reference's hook (its pure-torch train.py from the staged copy under
oracle/_ref, run on the CPU where its Hadamard matmul is the sequential FMA chain this package's kernels reproduce):
  * the K fake quantization on groups of real indices (plain, left-padded, packed documents) is bit-identical;
  * a full 800h forward of a small model with the LFM3 module structure (padding + packing + a prefill boundary, both
    rules) gives the reference hook's logits, while differing clearly from stock attention;
  * backward through the STE gives finite gradients, also on padded rows."""
import copy
import importlib.util
import os

import pytest
import torch

import _lfm3_stub as stub

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TRAIN = os.path.join(ROOT, "oracle", "_ref", "lfm3_kv800", "train.py")


@pytest.fixture(scope="module")
def ref_train():
    if not os.path.exists(REF_TRAIN):
        pytest.skip("the reference package is not staged under oracle/_ref (oracle/stage_reference.py)")
    spec = importlib.util.spec_from_file_location("ref_lfm3_train_gpu", REF_TRAIN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def T():
    from lfm3_kv800 import train
    return train


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize("case", ["plain", "padded", "packed"])
def test_fq_k_bit_exact_vs_reference(ref_train, T, case):
    B, Tn = 2, 900
    g = torch.Generator().manual_seed(3)
    kp = (torch.randn(B, Tn, 4, 128, generator=g) * (1 + 3 * torch.rand(1, 1, 4, 128, generator=g))).bfloat16()
    kw = {}
    if case == "padded":
        am = torch.ones(B, Tn, dtype=torch.long)
        am[1, :123] = 0
        kw = dict(attention_mask=am)
    elif case == "packed":
        kw = dict(position_ids=torch.cat((torch.arange(600), torch.arange(300)))[None].expand(B, Tn))
    ref = ref_train._Layout(B, Tn, "cpu", "cache", **kw).fq_k(kp)
    kwd = {k: v.to(DEV) for k, v in kw.items()}
    got = T._Geometry(B, Tn, DEV, "cache", **kwd).fq_k(kp.to(DEV)).cpu()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def _batch():
    g = torch.Generator().manual_seed(9)
    x = torch.randint(0, 97, (2, 700), generator=g)
    am = torch.ones_like(x)
    am[1, :150] = 0                                              # row 1 left-padded
    return x, am


@pytest.mark.parametrize("rule", ["cache", "last128"])
def test_800h_forward_matches_reference_hook(ref_train, T, rule):
    torch.backends.cuda.matmul.allow_tf32 = False
    base = stub.make_model(5)
    ours_m, ref_m = copy.deepcopy(base).to(DEV), copy.deepcopy(base)
    x, am = _batch()
    ours = T.patch_for_training(ours_m, rule=rule)
    ref = ref_train.patch_for_training(ref_m, rule=rule)
    packed = torch.cat((torch.arange(400), torch.arange(300)))[None].expand(2, 700)
    try:
        with torch.no_grad():
            for kw, keep in ((dict(attention_mask=am), am.bool()), (dict(position_ids=packed), None)):
                kwd = {k: v.to(DEV) for k, v in kw.items()}
                lo, lr = ours_m(x.to(DEV), **kwd).logits.cpu(), ref_m(x, **kw).logits
                if keep is not None:                             # logits of padding columns are not compared
                    lo, lr = lo[keep], lr[keep]
                err = _rel(lo, lr)
                with ours.using("stock"):
                    ls = ours_m(x.to(DEV), **kwd).logits.cpu()
                if keep is not None:
                    ls = ls[keep]
                effect = _rel(lo, ls)
                # the two models' fp32 projections differ in the last bits (CPU vs CUDA), which now and then moves
                # a key across a 2-bit / 1-bit decision; the K fake quant itself is bit-exact (test above).  The bar:
                # within 1e-2 and a small fraction of what the 800h cache changes relative to stock attention.
                assert err < 1e-2 and err < 0.1 * effect, \
                    f"{rule} {list(kw)}: logits rel {err:.2e} vs the reference hook (800h vs stock: {effect:.2e})"
            with ours.prefill(384), ref.prefill(384):
                lo = ours_m(x.to(DEV)).logits.cpu()
                lr = ref_m(x).logits
            assert _rel(lo, lr) < 1e-2
    finally:
        ours.remove()
        ref.remove()


def test_backward_finite_through_padding(T):
    m = stub.make_model(6, device=DEV)
    x, am = _batch()
    x, am = x.to(DEV), am.to(DEV)
    hook = T.patch_for_training(m)
    try:
        labels = x.masked_fill(am == 0, -100)
        loss = m(x, attention_mask=am, labels=labels).loss
        loss.backward()
        grads = [p.grad for p in m.parameters() if p.requires_grad]
        assert all(g is not None and torch.isfinite(g).all() for g in grads)
        for l in T.QUANT_LAYERS:
            assert m.model.layers[l].self_attn.k_proj.weight.grad.abs().sum() > 0
    finally:
        hook.remove()
