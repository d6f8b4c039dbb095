"""The training-side fake quant on CUDA against the reference's train.fake_quant_k / fake_quant_v (golden fixtures)
and the oracle: bit-exact for K and V; equal to the cache round trip (reference tests/test_train_hook.py:92-106);
straight-through gradients."""
import numpy as np
import pytest
import torch

import inputs as I
from oracle import oracle as O

pytestmark = pytest.mark.gpu
FG = np.load(I.__file__.replace("inputs.py", "fakequant.npz"))
DEV = "cuda"


@pytest.fixture(scope="module")
def kt():
    from lfm3_kv800 import train as m
    return m


@pytest.mark.parametrize("kind", ["normal", "outlier", "edge"])
def test_fake_quant_matches_reference(kt, kind):
    k, v = I.quant_inputs(kind, 2, seed=3)
    kf = torch.from_numpy(I.bf16_to_f32(k).reshape(2, 256, 512).copy()).to(DEV)
    vf = torch.from_numpy(I.bf16_to_f32(v).copy()).to(DEV)
    fk = kt.fake_quant_k(kf).cpu().numpy()
    fv = kt.fake_quant_v(vf, kt.hadamard(128, DEV)).cpu().numpy()
    assert I.digest(fk) == str(FG[f"{kind}_k_sha"])
    assert I.digest(fv) == str(FG[f"{kind}_v_sha"])


def test_fake_quant_equals_cache_round_trip(kt):
    from lfm3_kv800 import kv800
    k, v = I.quant_inputs("parity", 3, seed=2)
    kb = torch.from_numpy(k.view(np.int16)).view(torch.bfloat16).to(DEV)
    vb = torch.from_numpy(v.view(np.int16)).view(torch.bfloat16).to(DEV)
    kd, vd = kv800.dequantize_blocks(kv800.quantize_blocks(kb, vb))
    fk = kt.fake_quant_k(kb.float().reshape(3, 256, 512)).reshape(3, 256, 4, 128).to(torch.bfloat16)
    assert torch.equal(fk, kd)
    fv = kt.fake_quant_v(vb.float())
    assert torch.equal(fv, vd)          # same FMA chain on both sides: exact, stronger than the reference's allclose


def test_fake_quant_many_groups_vs_oracle(kt):
    rs = np.random.RandomState(4)
    x = (rs.standard_normal((5, 256, 512)) * rs.uniform(0.01, 30, (1, 1, 512))).astype(np.float32)
    v = (rs.standard_normal((777, 4, 128)) * 3).astype(np.float32)
    np.testing.assert_array_equal(kt.fake_quant_k(torch.from_numpy(x).to(DEV)).cpu().numpy(), O.fake_quant_k(x))
    np.testing.assert_array_equal(kt.fake_quant_v(torch.from_numpy(v).to(DEV)).cpu().numpy(), O.fake_quant_v(v))


def test_ste_gradient_is_identity(kt):
    x = torch.randn(2, 256, 512, device=DEV, requires_grad=True)
    y = kt.ste(x, kt.fake_quant_k)
    assert torch.equal(y.detach(), kt.fake_quant_k(x.detach()))
    (y * 3).sum().backward()
    assert torch.equal(x.grad, torch.full_like(x, 3.0))
