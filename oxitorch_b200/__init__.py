"""oxitorch_b200 -- B200-native (sm_100a) backend for oxitorch's memory-bound
layer path: RMSNorm / LayerNorm(+GELU) / softmax / log_softmax / cross-entropy /
SiLU-SwiGLU / registry elementwise ops / dim and whole-tensor reductions /
embedding gather and its duplicate-id VJP.

The product is ``liboxicuda.so`` (C ABI, ``include/oxicuda.h``); this package
is the host-side mirror of the reference's operator surface on top of it.
"""

from . import _native  # noqa: F401
from . import functional  # noqa: F401

__all__ = ["functional"]
