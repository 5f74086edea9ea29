"""A tiny causal LM used as the workload of the whole-path parity tests.

The capture layer class is a parameter, so the same architecture runs with
the reference's GCLinear (to record golden outputs) and with
opus_b200.layers.GCLinear (the path under test).  The forward signature is
the one the selection code calls: model(input_seq, target_seq=None,
sliding_window_num_blocks=None) returns logits, or the mean token loss when
targets are given.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F


class TinyLM(nn.Module):
    def __init__(self, linear_cls, vocab: int = 256, d: int = 64, hidden: int = 128, n_layers: int = 2,
                 last_bias: bool = True):
        super().__init__()
        self.vocab, self.d = vocab, d
        self.embed = nn.Embedding(vocab, d)
        self.fc1 = nn.ModuleList([linear_cls(d, hidden, bias=False) for _ in range(n_layers)])
        self.fc2 = nn.ModuleList([linear_cls(hidden, d, bias=(last_bias and i == n_layers - 1))
                                  for i in range(n_layers)])
        self.lm_head = nn.Linear(d, vocab, bias=False)  # not a capture layer, as in the reference model

    def forward(self, input_seq, target_seq=None, sliding_window_num_blocks=None):
        if input_seq.ndim == 1:
            input_seq = input_seq[None]
        x = self.embed(input_seq)
        T = x.shape[1]
        pos = torch.arange(1, T + 1, device=x.device, dtype=x.dtype).view(1, T, 1)
        x = torch.cumsum(x, dim=1) / pos  # causal token mixing
        for fc1, fc2 in zip(self.fc1, self.fc2):
            x = x + fc2(F.gelu(fc1(F.rms_norm(x, (self.d,)))))
        logits = self.lm_head(F.rms_norm(x, (self.d,)))
        if target_seq is not None:
            return F.cross_entropy(logits.float().view(-1, self.vocab), target_seq.reshape(-1))
        return logits


class SmallGPT2(nn.Module):
    """GPT-2-small-wide blocks (d 768, 12 heads, MLP 3072, vocab 50257, T up to 1024).

    Four capture layers per block (qkv, attention out, MLP in, MLP out), learned
    positions, pre-LayerNorm, causal attention, tanh GELU, the head tied to the
    token embedding.  Weights come from torch.manual_seed before construction,
    so the reference run and the run under test build the same model.
    """

    def __init__(self, linear_cls, n_layer: int = 2, vocab: int = 50257, d: int = 768, n_head: int = 12,
                 mlp: int = 3072, ctx: int = 1024):
        super().__init__()
        self.vocab, self.d, self.n_head = vocab, d, n_head
        self.wte, self.wpe = nn.Embedding(vocab, d), nn.Embedding(ctx, d)
        self.ln1 = nn.ModuleList([nn.LayerNorm(d) for _ in range(n_layer)])
        self.ln2 = nn.ModuleList([nn.LayerNorm(d) for _ in range(n_layer)])
        self.qkv = nn.ModuleList([linear_cls(d, 3 * d, bias=True) for _ in range(n_layer)])
        self.proj = nn.ModuleList([linear_cls(d, d, bias=True) for _ in range(n_layer)])
        self.fc = nn.ModuleList([linear_cls(d, mlp, bias=True) for _ in range(n_layer)])
        self.fc_proj = nn.ModuleList([linear_cls(mlp, d, bias=True) for _ in range(n_layer)])
        self.ln_f = nn.LayerNorm(d)
        with torch.no_grad():
            for m in [*self.qkv, *self.proj, *self.fc, *self.fc_proj]:
                m.weight.normal_(0.0, 0.02)
                m.bias.zero_()
            self.wte.weight.normal_(0.0, 0.02)
            self.wpe.weight.normal_(0.0, 0.01)

    def forward(self, input_seq, target_seq=None, sliding_window_num_blocks=None):
        if input_seq.ndim == 1:
            input_seq = input_seq[None]
        B, T = input_seq.shape
        x = self.wte(input_seq) + self.wpe(torch.arange(T, device=input_seq.device))
        for i in range(len(self.qkv)):
            q, k, v = self.qkv[i](self.ln1[i](x)).split(self.d, dim=2)
            q, k, v = (t.view(B, T, self.n_head, -1).transpose(1, 2) for t in (q, k, v))
            att = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, self.d)
            x = x + self.proj[i](att)
            x = x + self.fc_proj[i](F.gelu(self.fc[i](self.ln2[i](x)), approximate="tanh"))
        logits = F.linear(self.ln_f(x), self.wte.weight)
        if target_seq is not None:
            return F.cross_entropy(logits.float().view(-1, self.vocab), target_seq.reshape(-1))
        return logits

    def weight_checksum(self) -> float:
        return float(sum(p.detach().double().sum().item() + p.detach().double().abs().sum().item()
                         for p in self.parameters()))


class SmallQwen3(nn.Module):
    """Qwen3-style blocks: RMSNorm, grouped-query attention with per-head q/k RMSNorm and
    RoPE, SwiGLU MLP; seven capture layers per block (q, k, v, o, gate, up, down), the head
    tied to the token embedding.  Weights come from torch.manual_seed before construction.
    """

    def __init__(self, linear_cls, n_layer: int = 1, vocab: int = 151936, d: int = 2048, n_head: int = 16,
                 n_kv: int = 8, head_dim: int = 128, mlp: int = 6144, theta: float = 1e6):
        super().__init__()
        self.vocab, self.d, self.n_head, self.n_kv, self.head_dim, self.theta = vocab, d, n_head, n_kv, head_dim, theta
        self.embed = nn.Embedding(vocab, d)
        mk = lambda i, o: nn.ModuleList([linear_cls(i, o, bias=False) for _ in range(n_layer)])  # noqa: E731
        self.q, self.k, self.v = mk(d, n_head * head_dim), mk(d, n_kv * head_dim), mk(d, n_kv * head_dim)
        self.o = mk(n_head * head_dim, d)
        self.gate, self.up, self.down = mk(d, mlp), mk(d, mlp), mk(mlp, d)
        with torch.no_grad():
            for m in [*self.q, *self.k, *self.v, *self.o, *self.gate, *self.up, *self.down]:
                m.weight.normal_(0.0, 0.02)
            self.embed.weight.normal_(0.0, 0.02)

    def _rope(self, x):
        T, hd = x.shape[1], self.head_dim
        inv = self.theta ** (-torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd)
        ang = torch.arange(T, device=x.device, dtype=torch.float32)[:, None] * inv[None, :]
        cos, sin = torch.cos(ang).repeat(1, 2)[None, :, None, :], torch.sin(ang).repeat(1, 2)[None, :, None, :]
        x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
        return x * cos.to(x.dtype) + torch.cat([-x2, x1], dim=-1) * sin.to(x.dtype)

    def forward(self, input_seq, target_seq=None, sliding_window_num_blocks=None):
        if input_seq.ndim == 1:
            input_seq = input_seq[None]
        B, T = input_seq.shape
        x = self.embed(input_seq)
        hd = self.head_dim
        for i in range(len(self.q)):
            h = F.rms_norm(x, (self.d,))
            q = F.rms_norm(self.q[i](h).view(B, T, self.n_head, hd), (hd,))
            k = F.rms_norm(self.k[i](h).view(B, T, self.n_kv, hd), (hd,))
            v = self.v[i](h).view(B, T, self.n_kv, hd)
            q, k = self._rope(q), self._rope(k)
            rep = self.n_head // self.n_kv
            k, v = k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)
            att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                 is_causal=True)
            x = x + self.o[i](att.transpose(1, 2).reshape(B, T, self.n_head * hd))
            h = F.rms_norm(x, (self.d,))
            x = x + self.down[i](F.silu(self.gate[i](h)) * self.up[i](h))
        logits = F.linear(F.rms_norm(x, (self.d,)), self.embed.weight)
        if target_seq is not None:
            return F.cross_entropy(logits.float().view(-1, self.vocab), target_seq.reshape(-1))
        return logits

    def weight_checksum(self) -> float:
        return float(sum(p.detach().double().sum().item() + p.detach().double().abs().sum().item()
                         for p in self.parameters()))


def lora_factory(cls, r: int = 4, alpha: int = 8):
    """TinyLM capture-layer constructor for a LoRA linear of rank r (LoRALinear has no bias)."""

    def make(in_features: int, out_features: int, bias: bool = False):
        return cls(in_features, out_features, r=r, lora_alpha=alpha)

    return make


class MuonLike:
    """Minimal optimizer exposing a momentum group and momentum buffers (Muon's state layout)."""

    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95):
        self.param_groups = [dict(params=list(params), lr=lr, momentum=momentum)]
        self.state: dict = {}


class ProxyLoader:
    """Validation loader stand-in holding one pinned proxy batch."""

    def __init__(self, batch):
        self._fixed_batch = batch


def zipf_tokens(rng: np.random.Generator, n: int, T: int, vocab: int, a: float = 1.1) -> np.ndarray:
    """Token ids drawn Zipf(a) over the vocabulary (rank = id), truncated at vocab."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-a)
    p /= p.sum()
    return rng.choice(vocab, size=(n, T), p=p).astype(np.int64)


def state_to_numpy(model: nn.Module) -> dict:
    return {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}


def load_numpy_state(model: nn.Module, arrays: dict, prefix: str = "w/") -> None:
    sd = {k[len(prefix):]: torch.from_numpy(np.asarray(v)) for k, v in arrays.items() if k.startswith(prefix)}
    model.load_state_dict({k: sd[k].to(model.state_dict()[k].dtype) for k in model.state_dict()})
