"""LoRA layers with activation capture (drop-in for OPUS/layers/lora_layers.py).

``LoRALinear`` adds a rank-r update B A (scaled by alpha / r) to a frozen
dense weight; ``GCLoRALinear`` additionally records the layer input and output
with a forward hook and factors the gradients of both LoRA matrices into
(dL/dZ, A) pairs the selection kernels consume (lora_layers.py:98-135).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class LoRALayer:
    """Shared LoRA hyper-parameters (lora_layers.py:18-35)."""

    def __init__(self, r: int, lora_alpha: int, lora_dropout: float, merge_weights: bool):
        self.r = r
        self.lora_alpha = lora_alpha
        self.lora_dropout = nn.Dropout(p=lora_dropout) if lora_dropout > 0.0 else (lambda x: x)
        self.merged = False
        self.merge_weights = merge_weights


class LoRALinear(nn.Linear, LoRALayer):
    """Dense layer with a low-rank trainable update (lora_layers.py:38-95)."""

    def __init__(self, in_features: int, out_features: int, r: int = 0, lora_alpha: int = 1,
                 lora_dropout: float = 0.0, fan_in_fan_out: bool = False, merge_weights: bool = True, **kwargs):
        nn.Linear.__init__(self, in_features, out_features, bias=False, **kwargs)
        LoRALayer.__init__(self, r=r, lora_alpha=lora_alpha, lora_dropout=lora_dropout, merge_weights=merge_weights)
        self.fan_in_fan_out = fan_in_fan_out
        if r > 0:
            self.lora_A = nn.Parameter(self.weight.new_zeros((r, in_features)))
            self.lora_B = nn.Parameter(self.weight.new_zeros((out_features, r)))
            self.scaling = self.lora_alpha / self.r
            self.weight.requires_grad = False
        self.reset_parameters()
        if fan_in_fan_out:
            self.weight.data = self.weight.data.transpose(0, 1)

    def _oriented(self, w: torch.Tensor) -> torch.Tensor:
        return w.transpose(0, 1) if self.fan_in_fan_out else w

    def reset_parameters(self) -> None:
        nn.Linear.reset_parameters(self)
        if hasattr(self, "lora_A"):
            nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
            nn.init.zeros_(self.lora_B)

    def train(self, mode: bool = True):
        nn.Linear.train(self, mode)
        if not self.merge_weights or self.merged != mode:
            return self
        # training un-merges the low-rank update, inference folds it into weight
        if self.r > 0:
            delta = self._oriented(self.lora_B @ self.lora_A) * self.scaling
            if mode:
                self.weight.data -= delta
            else:
                self.weight.data += delta
        self.merged = not mode
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = F.linear(x, self._oriented(self.weight), bias=self.bias)
        if self.r > 0 and not self.merged:
            out += (self.lora_dropout(x) @ self.lora_A.transpose(0, 1) @ self.lora_B.transpose(0, 1)) * self.scaling
        return out


class GCLoRALinear(LoRALinear):
    """LoRA layer whose LoRA-parameter gradients factor into (dL/dZ, A) pairs."""

    def __init__(self, in_features: int, out_features: int, r: int = 0, lora_alpha: int = 1,
                 lora_dropout: float = 0.0, fan_in_fan_out: bool = False, merge_weights: bool = True, **kwargs):
        super().__init__(in_features, out_features, r=r, lora_alpha=lora_alpha, lora_dropout=lora_dropout,
                         fan_in_fan_out=fan_in_fan_out, merge_weights=merge_weights, **kwargs)
        self.layer_type = "GC_Linear_LoRA"
        self.register_forward_hook(self.capture_hook)

    def capture_hook(self, module, input, output):  # noqa: A002 - hook signature
        self.layer_input = input[0]
        self.pre_activation = output

    def pe_grad_gradcomp(self, deriv_pre_activ: torch.Tensor, per_sample: bool = True):
        """[(dL/dO B, a), (dL/dO, a A^T)] for lora_A and lora_B (lora_layers.py:120-135)."""
        a = self.layer_input.to(self.lora_A.dtype)
        g = (deriv_pre_activ * deriv_pre_activ.shape[0]).to(self.lora_B.dtype)
        return [(torch.matmul(g, self.lora_B), a), (g, torch.matmul(a, self.lora_A.T))]
