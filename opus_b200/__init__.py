"""OPUS per-iteration data selection on B200 (sm_100a).

Drop-in for the reference package ``OPUS`` (gszfwsb/OPUS): ``opus_b200.layers``
mirrors ``OPUS.layers`` and ``opus_b200.train`` mirrors ``OPUS.train``.  The
numeric work runs in libopus_b200.so (C ABI in include/opus_b200.h).
``install_as_OPUS()`` registers the package under the reference's module
names so unmodified ``import OPUS.train`` call sites resolve here.
"""
import sys

__version__ = "1.0.0"


def install_as_OPUS() -> None:
    """Make ``import OPUS``, ``OPUS.layers`` and ``OPUS.train`` resolve to this package."""
    from . import layers, train
    from .layers import linear, lora_layers
    from .train import data_selection, random_projection

    mod = sys.modules[__name__]
    sys.modules["OPUS"] = mod
    sys.modules["OPUS.layers"] = layers
    sys.modules["OPUS.layers.linear"] = linear
    sys.modules["OPUS.layers.lora_layers"] = lora_layers
    sys.modules["OPUS.train"] = train
    sys.modules["OPUS.train.data_selection"] = data_selection
    sys.modules["OPUS.train.random_projection"] = random_projection
