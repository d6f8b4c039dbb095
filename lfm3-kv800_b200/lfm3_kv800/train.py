"""Training side of the 800h cache on the CUDA backend: the fake quantization that puts the 800h cache in the loop of
an SFT / RL forward, and the model hook that applies it to an LFM3-1.7B HF model (the reference's train.py,
lfm3_kv800/train.py, same names and behaviour).

    hook = patch_for_training(model)               # any wrapper of an LFM3 HF model: PEFT, DDP, ...
    loss = model(input_ids=x, attention_mask=m, labels=y).loss   # layers 2/6/10/14/18/22 attend through 800h
    hook.set_mode("stock")                         # the unmodified attention, same weights
    with hook.prefill(prompt_width): ...           # RL: query columns < prompt_width were prefilled by the sampler
    hook.remove()                                  # puts the model back exactly

The ops (CUDA tensors only; no CPU path):
  fake_quant_k(x): x (..., G, 256, C) fp32 pre-RoPE keys in groups of 256 tokens -> dequantized 800h K (fp32): per
      (group, channel) 2-bit codes, lo and scale (hi - lo) / 3 rounded to fp8 e4m3 (train.py:82-89).
  fake_quant_v(v, H): v (..., 4, 128) fp32 values -> per-head Hadamard, 1 bit per dim over 2 groups of 256 dims per
      token, fp8 lo and scale hi - lo, rotated back (train.py:92-100).
  Both are bit-identical to the reference's torch functions on CPU (the Hadamard as the sequential fp32 FMA chain) and
  therefore to the cache round trip dequantize_blocks(quantize_blocks(.)).
  ste(x, fq): forward fq(x), gradient straight through (train.py:238-242).

The hook (train.py:245-404): on the full-attention layers 6, 10, 14, 22 every query sees each older key either
exact or through its 800h quantize-dequantize (K per aligned 256-token group, pre-RoPE, then rotated; V per token),
in one SDPA over [exact K/V | 800h K/V] with a [T, 2T] boolean mask; layers 2 and 18 see 4 sink tokens plus the last
256.  Which keys are quantized follows the cache's flush rule (rule="cache": the query at real index i reads key j
quantized iff j < 256 ((i + 1 - 128) // 256)) or the probe rule (rule="last128": keys at least 128 back in a
complete group).  Real indices are counted per row on its attention_mask and per packed document (position_ids that
restart at 0); padding keys are never visible and pad query rows see only themselves.  Query columns marked as
prefill see all keys exact on the quantized layers.  Gradients pass straight through the quantization."""
import contextlib
import ctypes
import sys
import weakref
from collections import OrderedDict

import torch
import torch.nn.functional as F

from . import _lib
from .kv800 import BLK, LAG, NSINK, WIN, _cuda, _ptr, _stream, hadamard

QUANT_LAYERS, WINDOW_LAYERS = (6, 10, 14, 22), (2, 18)
F8 = torch.float8_e4m3fn
MODES, RULES = ("800h", "stock"), ("cache", "last128")

__all__ = ["patch_for_training", "KV800TrainHook", "fake_quant_k", "fake_quant_v", "ste", "hadamard",
           "apply_transformers_compat", "QUANT_LAYERS", "WINDOW_LAYERS", "BLK", "LAG", "NSINK", "WIN"]


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


# ---------------------------------------------------------------- per-forward geometry (train.py:115-226)
_MASK_CACHE: "OrderedDict" = OrderedDict()   # (T, rule, kind, device) -> mask of an unpadded, unpacked batch
_MASK_CACHE_SIZE = 8                          # RL sees many lengths; keep a few


def _cached_mask(key, make):
    m = _MASK_CACHE.get(key)
    if m is None:
        m = _MASK_CACHE[key] = make()
        while len(_MASK_CACHE) > _MASK_CACHE_SIZE:
            _MASK_CACHE.popitem(last=False)
    else:
        _MASK_CACHE.move_to_end(key)
    return m


class _Geometry:
    """Where every column of one forward sits: its real index within its document (padding and packed documents
    removed), which keys it may see exact or quantized, and how the pre-RoPE keys are grouped into 256-token groups
    of real indices for the K fake quantization.  Built once per forward and shared by the patched layers (attached
    to the forward's rotary cos tensor, so gradient-checkpoint recomputation finds the same one).

    The plain case (no padding, no packing, no prefill columns) keeps one layout for the whole batch, and its masks
    are cached by length.  Otherwise, per row: valid = attention_mask, doc = index of the packed document (a column
    whose position_id is not the previous one + 1 starts a document), r = number of valid columns of the same
    document before this one.  Documents are laid out at 256-aligned offsets of a compact buffer for the K groups."""

    def __init__(self, B, T, device, rule, attention_mask=None, position_ids=None, prefill=None):
        self.B, self.T, self.dev, self.rule = B, T, device, rule
        self.masks = {}
        valid = doc = pf = None
        if attention_mask is not None:
            am = attention_mask.to(device)
            if tuple(am.shape) != (B, T):
                raise ValueError(f"800h: attention_mask must be 2D (batch, seq) = {(B, T)}, got {tuple(am.shape)}")
            if not bool(am.bool().all()):
                valid = am.bool()
        if position_ids is not None and T > 1:
            p = position_ids.to(device).expand(B, T)
            starts = torch.ones(B, T, dtype=torch.bool, device=device)
            starts[:, 1:] = p[:, 1:] != p[:, :-1] + 1
            if bool(starts[:, 1:].any()):
                doc = starts.long().cumsum(1) - 1
        if prefill is not None:
            bound = torch.as_tensor(prefill, device=device).long().reshape(-1)
            if bound.numel() not in (1, B):
                raise ValueError(f"800h: prefill boundary must be an int or a ({B},) tensor, got {bound.numel()} "
                                 f"values")
            pf = torch.arange(T, device=device)[None] < bound.expand(B)[:, None]
            if not bool(pf.any()):
                pf = None
        self.plain = valid is None and doc is None and pf is None
        if self.plain:
            self.Tc = -(-T // BLK) * BLK
            return
        if valid is None:
            valid = torch.ones(B, T, dtype=torch.bool, device=device)
        if doc is None:
            doc = torch.zeros(B, T, dtype=torch.long, device=device)
        col = torch.arange(T, device=device).expand(B, T)
        first = torch.ones(B, T, dtype=torch.bool, device=device)
        first[:, 1:] = doc[:, 1:] != doc[:, :-1]
        start_col = torch.where(first, col, torch.zeros_like(col)).cummax(1).values      # first column of the doc
        vcount = valid.long().cumsum(1) - valid.long()                                   # valid columns before
        r = vcount - vcount.gather(1, start_col)
        ndoc = int(doc.max()) + 1
        length = torch.zeros(B, ndoc, dtype=torch.long, device=device).scatter_add_(1, doc, valid.long())
        span = (length + BLK - 1) // BLK * BLK
        base = span.cumsum(1) - span                                                     # doc offsets, 256-aligned
        slot = base.gather(1, doc) + r
        self.Tc = max(BLK, int(span.sum(1).max()))
        self.to_compact = torch.where(valid, slot, torch.full_like(slot, self.Tc))      # pads -> a dump row
        self.from_compact = torch.where(valid, slot, torch.zeros_like(slot)).clamp_max(self.Tc - 1)
        self.valid, self.doc, self.r, self.pf = valid, doc, r, pf
        self.complete = length.gather(1, doc) >= (r // BLK + 1) * BLK                   # the key's group is full

    # ---- K fake quantization on groups of real indices
    def fq_k(self, kp):
        """kp (B, T, 4, 128) pre-RoPE keys -> their 800h quantize-dequantize (same dtype), groups of 256 real tokens
        per document (a document's incomplete last group is padded with zeros, and never read quantized)."""
        B, T = kp.shape[:2]
        x = kp.detach().to(torch.bfloat16).float().reshape(B, T, -1)
        C = x.shape[-1]
        if self.plain:
            xp = F.pad(x, (0, 0, 0, self.Tc - T)) if self.Tc != T else x
            y = fake_quant_k(xp.reshape(B, self.Tc // BLK, BLK, C)).reshape(B, self.Tc, C)[:, :T]
        else:
            buf = x.new_zeros(B, self.Tc + 1, C)
            buf.scatter_(1, self.to_compact[..., None].expand(B, T, C), x)
            y = fake_quant_k(buf[:, :self.Tc].reshape(B, self.Tc // BLK, BLK, C)).reshape(B, self.Tc, C)
            y = y.gather(1, self.from_compact[..., None].expand(B, T, C))
        return y.to(torch.bfloat16).to(kp.dtype).reshape(kp.shape)

    # ---- masks: "win" (T, T) for layers 2 / 18, "quant" (T, 2T) = [exact | quantized] for 6 / 10 / 14 / 22
    def mask(self, kind):
        m = self.masks.get(kind)
        if m is None:
            if self.plain:
                m = _cached_mask((self.T, self.rule, kind, str(self.dev)), lambda: self._plain_mask(kind))
            else:
                m = self._general_mask(kind)
            self.masks[kind] = m
        return m

    def _plain_mask(self, kind):
        T = self.T
        i = torch.arange(T, device=self.dev)[:, None]
        j = torch.arange(T, device=self.dev)[None, :]
        seen = j <= i
        if kind == "win":
            return (seen & ((j > i - WIN) | (j < NSINK)))[None, None]
        if self.rule == "cache":
            quant = seen & (j < (i + 1 - LAG).clamp_min(0) // BLK * BLK)
        else:
            quant = seen & (j <= i - LAG) & ((j // BLK + 1) * BLK <= T)
        return torch.cat((seen & ~quant, quant), 1)[None, None]

    def _general_mask(self, kind):
        T = self.T
        ri, rj = self.r[:, :, None], self.r[:, None, :]
        seen = torch.ones(T, T, dtype=torch.bool, device=self.dev).tril()[None]
        seen = seen & self.valid[:, None, :] & (self.doc[:, :, None] == self.doc[:, None, :])
        own = torch.eye(T, dtype=torch.bool, device=self.dev)[None] & ~self.valid[:, :, None]   # pad query rows
        if kind == "win":
            return ((seen & ((rj > ri - WIN) | (rj < NSINK))) | own)[:, None]
        if self.rule == "cache":
            bound = (ri + 1 - LAG).clamp_min(0) // BLK * BLK
            if self.pf is not None:
                bound = bound.masked_fill(self.pf[:, :, None], 0)
            quant = seen & (rj < bound)
        else:
            quant = seen & (rj <= ri - LAG) & self.complete[:, None, :]
            if self.pf is not None:
                quant = quant & ~self.pf[:, :, None]
        return torch.cat(((seen & ~quant) | own, quant), 2)[:, None]


# ---------------------------------------------------------------- the hook (train.py:229-404)
def _backbone(model):
    """The LFM3 backbone inside any wrapper: the module with `layers`, `rotary_emb` and config.layer_types."""
    for mod in model.modules():
        if hasattr(mod, "layers") and hasattr(mod, "rotary_emb") and hasattr(getattr(mod, "config", None),
                                                                            "layer_types"):
            return mod
    raise ValueError("no LFM3 backbone (a module with .layers, .rotary_emb and config.layer_types) in the model")


_HADAMARD = {}


def _hadamard_on(device):
    key = str(device)
    if key not in _HADAMARD:
        _HADAMARD[key] = hadamard(128, device)
    return _HADAMARD[key]


class KV800TrainHook:
    """Handle of patch_for_training.  mode "800h" | "stock"; rule "cache" (the vLLM cache's flush rule) | "last128"."""

    def __init__(self, model, mode="800h", rule="cache", fp32_rope=True):
        if rule not in RULES:
            raise ValueError(f"rule must be one of {RULES}, got {rule!r}")
        lm = _backbone(model)
        held = getattr(lm, "_kv800_hook", None)
        if held is not None and held() is not None:
            raise RuntimeError("this model is already patched; call .remove() on the existing hook first")
        types_ = lm.config.layer_types
        for l in QUANT_LAYERS + WINDOW_LAYERS:
            if l >= len(types_) or types_[l] != "full_attention":
                raise ValueError(f"layer {l} is {types_[l] if l < len(types_) else 'missing'}, not full_attention: "
                                 f"not the LFM3-1.7B layout the 800h cache is defined for")
        self.rule, self.mode = rule, None
        self._lm, self._prefill, self._seen = lm, None, None
        self.set_mode(mode)
        # vLLM computes the rotary frequencies in fp32; rebuild a rotary module loaded in lower precision
        self._rope_saved = None
        rot = lm.rotary_emb
        low = [b for n, b in rot.named_buffers() if n.endswith("inv_freq") and b.dtype != torch.float32]
        if fp32_rope and low:
            self._rope_saved = rot
            lm.rotary_emb = type(rot)(lm.config, device=low[0].device)
        self._patched = []
        for l in QUANT_LAYERS + WINDOW_LAYERS:
            attn = lm.layers[l].self_attn
            own = attn.__dict__.get("forward")              # an instance-level forward to put back on remove()
            attn.forward = self._forward_for(attn, l, attn.forward)
            self._patched.append((attn, own))
        self._pre = lm.register_forward_pre_hook(self._capture, with_kwargs=True)
        lm._kv800_hook = weakref.ref(self)

    # ---- public API (train.py:294-352)
    def set_mode(self, mode):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
        self.mode = mode
        return self

    @contextlib.contextmanager
    def using(self, mode):
        """`with hook.using("stock"): ...` switches the mode for the block."""
        before = self.mode
        self.set_mode(mode)
        try:
            yield self
        finally:
            self.mode = before

    @contextlib.contextmanager
    def prefill(self, boundary):
        """Query columns < boundary (an int, or one per row) were computed by the sampler's prefill: on the quantized
        layers they see every key exact."""
        before = self._prefill
        self._prefill = boundary
        try:
            yield self
        finally:
            self._prefill = before

    def set_prefill(self, boundary):
        """prefill() without the context manager; None clears it."""
        self._prefill = boundary
        return self

    def remove(self):
        """Original attention forwards and rotary module back, pre-hook gone."""
        if self._lm is None:
            return
        for attn, own in self._patched:
            if own is None:
                attn.__dict__.pop("forward", None)
            else:
                attn.forward = own
        self._patched = []
        self._pre.remove()
        if self._rope_saved is not None:
            self._lm.rotary_emb = self._rope_saved
            self._rope_saved = None
        self._lm._kv800_hook = None
        self._lm = None

    # ---- internals
    def _capture(self, module, args, kwargs):
        """Backbone pre-forward hook: remember the forward's mask / positions (and refuse what 800h mode can't do)."""
        names = ("input_ids", "attention_mask", "position_ids", "past_key_values")
        got = {k: v for k, v in zip(names, args)}
        got.update({k: kwargs[k] for k in names if k in kwargs})
        if self.mode == "800h":
            if got.get("past_key_values") is not None:
                raise RuntimeError("800h training mode runs full-sequence forwards only (no past_key_values / "
                                   "generate); sample with the vLLM plugin, or set_mode('stock') to generate in HF")
            am = got.get("attention_mask")
            if am is not None and not (isinstance(am, torch.Tensor) and am.ndim == 2):
                raise RuntimeError("800h training mode needs a 2D (batch, seq) attention_mask or None")
        self._seen = (got.get("attention_mask"), got.get("position_ids"), self._prefill)
        return None

    def _geometry(self, hidden, cos):
        tagged = getattr(cos, "_kv800_geometry", None)
        if tagged is not None and tagged[0] is self:
            return tagged[1]
        B, T = hidden.shape[:2]
        am, pos, pf = self._seen if self._seen is not None else (None, None, self._prefill)
        if am is not None and tuple(am.shape) != (B, T):
            am = None                                  # layers called on their own: no padding information
        if pos is not None and pos.shape[-1] != T:
            pos = None
        g = _Geometry(B, T, hidden.device, self.rule, am, pos, pf)
        try:
            cos._kv800_geometry = (self, g)
        except (AttributeError, RuntimeError):
            pass
        return g

    def _forward_for(self, attn, layer, original):
        rope = sys.modules[type(attn).__module__].apply_rotary_pos_emb
        hook = self

        def forward(hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kw):
            if hook.mode == "stock":
                return original(hidden_states, position_embeddings=position_embeddings,
                                attention_mask=attention_mask, past_key_values=past_key_values, **kw)
            B, T, _ = hidden_states.shape
            heads = (B, T, -1, attn.head_dim)
            cos, sin = position_embeddings
            geo = hook._geometry(hidden_states, cos)
            q = attn.q_norm(attn.q_proj(hidden_states).view(heads)).transpose(1, 2)
            k_pre = attn.k_norm(attn.k_proj(hidden_states).view(heads))           # (B, T, 4, 128), before RoPE
            v = attn.v_proj(hidden_states).view(heads)
            q_rot, k_rot = rope(q, k_pre.transpose(1, 2), cos, sin)
            v_t = v.transpose(1, 2)
            if layer in QUANT_LAYERS:
                H = _hadamard_on(hidden_states.device)
                k_q = ste(k_pre, geo.fq_k)
                v_q = ste(v, lambda x: fake_quant_v(x.to(torch.bfloat16).float(), H).to(torch.bfloat16).to(x.dtype))
                _, k_q_rot = rope(q, k_q.transpose(1, 2), cos, sin)
                keys, values = torch.cat((k_rot, k_q_rot), 2), torch.cat((v_t, v_q.transpose(1, 2)), 2)
                mask = geo.mask("quant")
            else:
                keys, values = k_rot, v_t
                mask = geo.mask("win")
            rep = attn.num_key_value_groups
            keys, values = keys.repeat_interleave(rep, 1), values.repeat_interleave(rep, 1)
            o = F.scaled_dot_product_attention(q_rot, keys.to(q_rot.dtype), values.to(q_rot.dtype), attn_mask=mask,
                                               scale=attn.scaling)
            gate = torch.sigmoid(attn.gate_proj(hidden_states)).unsqueeze(-1)
            return attn.o_proj((o.transpose(1, 2) * gate).reshape(B, T, -1)), None

        return forward


def patch_for_training(model, mode="800h", rule="cache", fp32_rope=True):
    """Patch an LFM3-1.7B HF model (or a PEFT / DDP / ... wrapper of it) so that its forward attends through the
    800h cache on layers 2, 6, 10, 14, 18, 22 (train.py:407-411).  Returns the KV800TrainHook."""
    return KV800TrainHook(model, mode=mode, rule=rule, fp32_rope=fp32_rope)


def apply_transformers_compat():
    """Config-parsing shims that some transformers 5.x releases need for the LFM3 remote code (train.py:414-433): the
    "conv" layer type is allowed, and a per-layer-type rope_parameters dict is standardized instead of converted.
    A no-op where those private symbols do not exist.  Call before from_pretrained."""
    try:
        import transformers.configuration_utils as cu
        from transformers.modeling_rope_utils import RotaryEmbeddingConfigMixin
    except ImportError:
        return
    remap = getattr(cu, "_LEGACY_LAYER_TYPE_REMAP", None)
    if isinstance(remap, dict):
        remap.pop("conv", None)
    allowed = getattr(cu, "ALLOWED_ATTN_LAYER_TYPES", None)
    if isinstance(allowed, tuple) and "conv" not in allowed:
        cu.ALLOWED_ATTN_LAYER_TYPES = allowed + ("conv",)
    mixin = RotaryEmbeddingConfigMixin
    if getattr(mixin, "_kv800_compat", False) or not hasattr(mixin, "convert_rope_params_to_dict"):
        return
    convert = mixin.convert_rope_params_to_dict

    def convert_per_type(self, **kw):
        rp = getattr(self, "rope_parameters", None)
        if isinstance(rp, dict) and any(isinstance(v, dict) for v in rp.values()):
            self._rope_type_labels = getattr(self, "_rope_type_labels", getattr(self, "_attention_layer_types", None))
            self.standardize_rope_params()
            return kw
        return convert(self, **kw)

    mixin.convert_rope_params_to_dict = convert_per_type
    mixin._kv800_compat = True
