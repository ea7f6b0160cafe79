"""The two loss entry points of functions/losses.py:8-67 (AndyBarcia/mask_loss)
on the B200 kernels: ``sigmoid_cross_entropy_loss`` and ``dice_loss``.

Same names, argument order and defaults.  The reference calls its Function
classes directly (``SigmoidCELossFunction(logits, ...)``) instead of through
``.apply``, and imports modules that do not exist, so its module cannot be
imported at all; here both entries go through ``.apply`` and autograd works.

``logits`` are ``(L, B, C, h, w)`` as the Functions take them (one loss per
layer, shape ``(L,)``) or ``(B, C, h, w)`` as the reference docstrings state
(a 0-d loss).  ``targets`` is the ``(B, H, W)`` integer label map with H, W
integer multiples of h, w.

Only the ``class_mapping=None`` path is provided: the multi-class mapping
variants are not part of the matching hot path.  ``implementation="python"``
selects the reference's CPU twins, which this package does not ship (it has
no CPU path); both raise ``ValueError``.
"""
from __future__ import annotations

import torch

from .semantic import DiceLossFunction, SigmoidCELossFunction


def _layers(logits: torch.Tensor):
    if logits.dim() == 4:
        return logits.unsqueeze(0), True
    if logits.dim() == 5:
        return logits, False
    raise ValueError("logits must be (B, C, h, w) or (L, B, C, h, w)")


def _check(class_mapping, implementation):
    if class_mapping is not None:
        raise ValueError("class_mapping is not supported by mask_loss_b200 (label maps only)")
    if implementation != "cuda":
        raise ValueError("mask_loss_b200 runs on CUDA only (implementation must be 'cuda')")


def sigmoid_cross_entropy_loss(logits, targets, class_mapping=None, num_masks=None,
                               implementation="cuda", scale=1.0):
    """Count-based sigmoid BCE of every class logit against its class's pixel
    counts (functions/losses.py:8-31 with class_mapping=None; the kernel is
    src/cuda/sigmoid_ce.cu)."""
    _check(class_mapping, implementation)
    x, squeeze = _layers(logits)
    out = SigmoidCELossFunction.apply(x, targets, num_masks, scale)
    return out[0] if squeeze else out


def dice_loss(logits, targets, smooth=1e-6, class_mapping=None, num_masks=None,
              implementation="cuda", scale=1.0):
    """Count-based dice loss consistent with nearest upsampling of the logits
    (functions/losses.py:34-67 with class_mapping=None; the kernel is
    src/cuda/dice_loss.cu)."""
    _check(class_mapping, implementation)
    x, squeeze = _layers(logits)
    out = DiceLossFunction.apply(x, targets, smooth, num_masks, scale)
    return out[0] if squeeze else out
