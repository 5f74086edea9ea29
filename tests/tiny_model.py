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
