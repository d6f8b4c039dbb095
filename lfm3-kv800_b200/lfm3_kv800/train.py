"""Training-side 800h ops on the CUDA backend: the fake quantization that puts the 800h cache in the loop of an SFT / RL
forward (the hot ops of the reference's train.py, lfm3_kv800/train.py:82-100,238-242).

    k_q = ste(k_pre_rope, fake_quant_k_tokens)    # forward = the cache's K quantize-dequantize, gradient = identity
    v_q = ste(v, lambda x: fake_quant_v(x, H))

fake_quant_k(x): x (..., G, 256, C) fp32 pre-RoPE keys in groups of 256 tokens -> dequantized 800h K (fp32): per
(group, channel) 2-bit codes, lo and scale (hi - lo) / 3 rounded to fp8 e4m3.
fake_quant_v(v, H): v (..., 4, 128) fp32 values -> per-head Hadamard, 1 bit per dim over 2 groups of 256 dims per
token, fp8 lo and scale hi - lo, rotated back.
Both are bit-identical to the reference's torch functions on CPU (the Hadamard as the sequential fp32 FMA chain) and
therefore to the cache round trip dequantize_blocks(quantize_blocks(.)).  CUDA tensors only; no CPU path.

The reference's model hook (patch_for_training, KV800TrainHook: HF monkey-patching, masks, packing) is model plumbing
around these ops and is not part of this package."""
import ctypes

import torch

from . import _lib
from .kv800 import BLK, LAG, NSINK, WIN, _cuda, _ptr, _stream, hadamard

QUANT_LAYERS, WINDOW_LAYERS = (6, 10, 14, 22), (2, 18)
F8 = torch.float8_e4m3fn

__all__ = ["fake_quant_k", "fake_quant_v", "ste", "hadamard", "QUANT_LAYERS", "WINDOW_LAYERS", "BLK", "LAG",
           "NSINK", "WIN"]


def fake_quant_k(x):
    """x (..., G, 256, C) fp32 pre-RoPE keys, groups of 256 tokens on dim -2 -> dequantized 800h K (fp32)."""
    _cuda(x, "fake_quant_k")
    if x.dim() < 2 or x.shape[-2] != BLK:
        raise ValueError(f"fake_quant_k: expected (..., G, 256, C), got {tuple(x.shape)}")
    if x.dtype != torch.float32:
        raise TypeError(f"fake_quant_k: expected float32, got {x.dtype}")
    x = x.contiguous()
    C = x.shape[-1]
    G = x.numel() // (BLK * C) if C else 0
    out = torch.empty_like(x)
    _lib.call("kv800_fake_quant_k", _ptr(x), G, C, _ptr(out), _stream(x.device))
    return out


def fake_quant_v(v, H=None):
    """v (..., 4, 128) fp32 values -> dequantized 800h V (fp32).  H is accepted for signature compatibility and must be
    hadamard(128): the kernel applies the normalized 128-point Hadamard itself."""
    _cuda(v, "fake_quant_v")
    if v.dim() < 2 or tuple(v.shape[-2:]) != (4, 128):
        raise ValueError(f"fake_quant_v: expected (..., 4, 128), got {tuple(v.shape)}")
    if v.dtype != torch.float32:
        raise TypeError(f"fake_quant_v: expected float32, got {v.dtype}")
    v = v.contiguous()
    out = torch.empty_like(v)
    _lib.call("kv800_fake_quant_v", _ptr(v), v.numel() // 512, _ptr(out), _stream(v.device))
    return out


def ste(x, fq):
    """Forward value exactly fq(x); gradient straight through (identity) -- the reference's _ste (train.py:238-242)."""
    with torch.no_grad():
        y = fq(x)
    return y + (x - x.detach())
