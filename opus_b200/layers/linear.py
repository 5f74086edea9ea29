"""Capture linear layer (stage 1 of the selection path).

``GCLinear`` is an ``nn.Linear`` that keeps, from its latest forward, the input
activations A (``layer_input``) and the output pre-activations Z
(``pre_activation``).  Differentiating the per-sample loss with respect to the
stored Z gives G = dL/dZ; (G, A) is all the selection kernels need, since the
per-sample weight gradient of a linear layer is G_b^T A_b.

Drop-in for OPUS.layers.linear.GCLinear (OPUS/layers/linear.py:14-126): same
constructor, attributes and methods, same scaling conventions.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class GCLinear(nn.Linear):
    """Linear layer that records its input and output for per-sample gradients."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__(in_features, out_features, bias)
        self.layer_input: torch.Tensor | None = None
        self.pre_activation: torch.Tensor | None = None
        self.name = "linear"
        self.has_bias = bias

    def forward(self, input: torch.Tensor) -> torch.Tensor:  # noqa: A002 - reference argument name
        # linear.py:35-39: keep A and Z of the latest call; Z stays in the graph.
        self.layer_input = input
        self.pre_activation = F.linear(input, self.weight, self.bias)
        return self.pre_activation

    def _scaled_grad(self, deriv_pre_activ: torch.Tensor) -> torch.Tensor:
        # The loss is a batch mean; multiplying by the batch size turns dL/dZ
        # into per-sample gradients (linear.py:56-57, 63-64, 118-119).
        return deriv_pre_activ * deriv_pre_activ.shape[0]

    def per_example_gradient(self, deriv_pre_activ: torch.Tensor):
        """Materialised per-sample (weight, bias) gradients (linear.py:41-68).

        2-D inputs give ([B, D_out, D_in], [B, D_out]); 3-D inputs follow the
        reference's permuted layout ([T, D_out, B] @ [T, B, D_in] -> [T, D_out, D_in]).
        """
        h = self.layer_input
        if h.dim() == 2:
            g = self._scaled_grad(deriv_pre_activ)
            return g.unsqueeze(2) * h.unsqueeze(1), g
        # Token-major layout, scaled by the leading (token) extent as in the
        # reference; unlike the reference, the caller's tensor is not modified.
        g = deriv_pre_activ.permute(1, 2, 0)
        g = g * g.size(0)
        return torch.bmm(g, h.transpose(0, 1)), g.sum(dim=-1)

    def pe_grad_sqnorm(self, deriv_pre_activ: torch.Tensor) -> torch.Tensor:
        """Squared norms of per-sample gradients (linear.py:70-101)."""
        h = self.layer_input
        if h.dim() == 2:
            g = self._scaled_grad(deriv_pre_activ)
            gz = g.pow(2).sum(1)
            return gz * h.pow(2).sum(1) + gz
        w, b = self.per_example_gradient(deriv_pre_activ)
        n = w.size(0)
        return w.pow(2).reshape(n, -1).sum(1) + b.pow(2).reshape(n, -1).sum(1)

    def pe_grad_gradcomp(self, deriv_pre_activ: torch.Tensor, per_sample: bool = True):
        """(dL/dZ * N, A): the factors of every per-sample gradient (linear.py:103-126).

        For 2-D inputs of a layer with bias, A gains a ones column so the bias
        gradient rides along; 3-D inputs keep A as is (the reference does the same).
        """
        h = self.layer_input
        g = self._scaled_grad(deriv_pre_activ)
        if h.dim() == 2 and self.has_bias:
            # default-dtype ones column, so bf16 inputs promote as in the reference
            h = torch.cat((h, torch.ones(h.size(0), 1, device=h.device)), dim=1)
        return g, h
