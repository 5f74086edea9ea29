"""Capture layers (drop-in for OPUS.layers, OPUS/layers/__init__.py:8-11)."""
from .linear import GCLinear
from .lora_layers import GCLoRALinear, LoRALinear

__all__ = ["GCLinear", "GCLoRALinear", "LoRALinear"]
