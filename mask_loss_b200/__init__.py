"""B200-native mask matching + loss (Mask2Former-style matcher and losses).

Drop-in for the hot path of AndyBarcia/mask_loss:

* ``mask_loss_b200.ops``       -- the ``mask_loss`` extension's op surface
                                   (same names and positional arguments);
* ``mask_loss_b200.functions`` -- the ``functions`` package's autograd
                                   Functions (same names and signatures);
* ``mask_loss_b200.parallel``  -- batch-by-image data parallelism over NCCL.

All compute runs in ``libmask_loss_b200.so`` (hand-written sm_100a CUDA behind
the C ABI of ``include/mask_loss_b200.h``).  There is no CPU fallback: using
an op without the library, or on CPU tensors, raises.
"""
from . import _lib  # noqa: F401
from . import ops  # noqa: F401
from .ops import check_status  # noqa: F401

__version__ = "0.1.0"


def library_path() -> str:
    return _lib.LIB_PATH
