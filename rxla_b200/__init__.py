"""rxla_b200 — B200 (sm_100a) kernels for rxla's W8 decode hot path.

The product is the C-ABI library ``librxla_b200.so`` (include/rxla_b200.h);
this package loads it (``_lib``), mirrors the reference operator surface on
torch device tensors (``nn``) and wraps the decoder runner (``decoder``).
There is no CPU fallback: without the built library every call raises.
"""
from ._lib import RxlaError, load  # noqa: F401

__version__ = "0.1.0"
