"""A small random-init model with the module structure the 800h training hook patches (the LFM3-1.7B HF remote
code's, as the reference's train.py reads it): a backbone with `layers`, `rotary_emb` and config.layer_types (24
layers, full attention at 2, 6, 10, 14, 18, 22), attention modules with q/k/v/o/gate projections, q/k RMS norms,
head_dim 128, 16 query / 4 KV heads, a sigmoid output gate per head, and a module-level apply_rotary_pos_emb (HF's
rotate-half form with 32 rotating frequencies, theta 1e6).  Test infrastructure only; the weights are not LFM3's."""
import types

import torch
import torch.nn.functional as F
from torch import nn

FULL = (2, 6, 10, 14, 18, 22)


def make_config(hidden=64, vocab=97):
    return types.SimpleNamespace(layer_types=["full_attention" if i in FULL else "conv" for i in range(24)],
                                 hidden_size=hidden, num_attention_heads=16, num_key_value_heads=4, head_dim=128,
                                 vocab_size=vocab)


class Rotary(nn.Module):
    def __init__(self, config, device=None, dtype=torch.float32):
        super().__init__()
        inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 128))
        self.register_buffer("inv_freq", torch.cat((inv, torch.zeros(32))).to(device=device, dtype=dtype),
                             persistent=False)

    def forward(self, x, position_ids):
        fr = position_ids[..., None].float() * self.inv_freq.float()
        emb = torch.cat((fr, fr), -1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


def rotate_half(x):
    return torch.cat((-x[..., 64:], x[..., :64]), -1)


def apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1):
    c, s = cos.unsqueeze(unsqueeze_dim), sin.unsqueeze(unsqueeze_dim)
    return q * c + rotate_half(q) * s, k * c + rotate_half(k) * s


class RMSNorm(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(x.dtype) * self.weight


class Attention(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        d, hd = cfg.hidden_size, cfg.head_dim
        self.head_dim = hd
        self.num_key_value_groups = cfg.num_attention_heads // cfg.num_key_value_heads
        self.scaling = hd ** -0.5
        self.q_proj = nn.Linear(d, cfg.num_attention_heads * hd, bias=False)
        self.k_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.v_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.gate_proj = nn.Linear(d, cfg.num_attention_heads, bias=False)      # one output gate per head
        self.o_proj = nn.Linear(cfg.num_attention_heads * hd, d, bias=False)
        self.q_norm, self.k_norm = RMSNorm(hd), RMSNorm(hd)

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None, **kw):
        B, T, _ = hidden_states.shape
        sh = (B, T, -1, self.head_dim)
        q = self.q_norm(self.q_proj(hidden_states).view(sh)).transpose(1, 2)
        k = self.k_norm(self.k_proj(hidden_states).view(sh)).transpose(1, 2)
        v = self.v_proj(hidden_states).view(sh).transpose(1, 2)
        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        k = k.repeat_interleave(self.num_key_value_groups, 1)
        v = v.repeat_interleave(self.num_key_value_groups, 1)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=self.scaling)
        gate = torch.sigmoid(self.gate_proj(hidden_states)).unsqueeze(-1)
        return self.o_proj((o.transpose(1, 2) * gate).reshape(B, T, -1)), None


class Layer(nn.Module):
    def __init__(self, cfg, i):
        super().__init__()
        self.norm = RMSNorm(cfg.hidden_size)
        if cfg.layer_types[i] == "full_attention":
            self.self_attn = Attention(cfg)
        else:
            self.conv = nn.Linear(cfg.hidden_size, cfg.hidden_size, bias=False)

    def forward(self, h, position_embeddings, attention_mask=None):
        x = self.norm(h)
        if hasattr(self, "self_attn"):
            return h + self.self_attn(x, position_embeddings=position_embeddings, attention_mask=attention_mask)[0]
        return h + 0.1 * torch.tanh(self.conv(x))


class Backbone(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([Layer(cfg, i) for i in range(24)])
        self.rotary_emb = Rotary(cfg)
        self.norm = RMSNorm(cfg.hidden_size)

    def forward(self, input_ids, attention_mask=None, position_ids=None, past_key_values=None):
        h = self.embed_tokens(input_ids)
        if position_ids is None:
            position_ids = torch.arange(input_ids.shape[1], device=input_ids.device)[None].expand_as(input_ids)
        pe = self.rotary_emb(h, position_ids)
        for layer in self.layers:
            h = layer(h, pe, attention_mask)
        return self.norm(h)


class CausalLM(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.model = Backbone(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)

    def forward(self, input_ids, attention_mask=None, position_ids=None, past_key_values=None, labels=None,
                use_cache=None):
        logits = self.lm_head(self.model(input_ids, attention_mask=attention_mask, position_ids=position_ids,
                                         past_key_values=past_key_values))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), labels[:, 1:].reshape(-1),
                                   ignore_index=-100)
        return types.SimpleNamespace(logits=logits, loss=loss)


def make_model(seed=0, device="cpu", dtype=torch.float32):
    torch.manual_seed(seed)
    m = CausalLM(make_config())
    for p in m.parameters():                      # projections large enough that attention is not uniform
        if p.dim() == 2:
            nn.init.normal_(p, std=0.6 / p.shape[1] ** 0.5)
    return m.to(device=device, dtype=dtype)
