"""qwen_megakernel_b200 -- persistent sm_100a decode megakernel for Qwen3-0.6B.

Drop-in for AlpinDale/qwen_megakernel's decode path: the same torch operators
(``torch.ops.qwen_megakernel_C.decode`` / ``generate_nosync``), the same
``Decoder`` API and the same bf16 weight / KV-cache layouts, on B200.

The native libraries are loaded on first use (``Decoder(...)`` or
``ops()``); there is no CPU fallback.
"""

from .model import Decoder, DecodeError, generate, load_weights, random_weights  # noqa: F401
from .batch import BatchDecoder, BatchError, BatchForward  # noqa: F401
from .weights import rope_tables  # noqa: F401
from ._native import ops, cdll  # noqa: F401

__all__ = [
    "load_weights",
    "random_weights",
    "rope_tables",
    "Decoder",
    "DecodeError",
    "BatchDecoder",
    "BatchError",
    "BatchForward",
    "generate",
    "ops",
    "cdll",
]
