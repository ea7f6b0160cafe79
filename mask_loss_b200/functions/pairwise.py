"""Pairwise cost Functions (forward-only, like the reference's).

PairwiseMaskLossFunction      functions/mask/pw_mask.py:21-115
PairwiseSigmoidCELossFunction functions/sigmoid/pw_sigmoid_ce.py:17-73
PairwiseDiceLossFunction      functions/dice/pw_dice_loss.py:15-57
PairwiseSigmoidLabelLossFunction functions/label/pw_sigmoid_label_loss.py:12-50
PairwiseSoftmaxLabelLossFunction functions/label/pw_softmax_label_loss.py:13-56
"""
from __future__ import annotations

from torch.autograd import Function

from .. import ops
from .matching import logits_for_kernels


def _gamma(v, default=0.0):
    g = default if v is None else float(v)
    if g < 0.0:
        raise ValueError("focal_gamma must be non-negative")
    return g


def _alpha(v, default=-1.0):
    if v is None:
        return default
    a = float(v)
    if not 0.0 <= a <= 1.0:
        raise ValueError("focal_alpha must be in [0, 1]")
    return a


def _ug(ug, ugmin):
    u = 1.0 if ug is None else float(ug)
    if u < 0.0:
        raise ValueError("uncertainty_gamma must be non-negative")
    m = 0.05 if ugmin is None else float(ugmin)
    if not 0.0 <= m <= 1.0:
        raise ValueError("uncertainty_gamma_min must be in [0, 1]")
    return u, m


class PairwiseMaskLossFunction(Function):
    @staticmethod
    def forward(ctx, mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale,
                dice_scale, cls_scale, background_index, uncertainty_gamma, uncertainty_gamma_min,
                normalize_uncertainty, mask_focal_gamma, mask_focal_alpha, cls_focal_gamma,
                cls_focal_alpha, label_loss="sigmoid"):
        assert mask_logits.shape[1] == mask_targets.shape[0], \
            "Batch size mismatch between logits and targets"
        mg = _gamma(mask_focal_gamma)
        ma = _alpha(mask_focal_alpha)
        cg = mg if cls_focal_gamma is None else _gamma(cls_focal_gamma)
        ca = ma if cls_focal_alpha is None else _alpha(cls_focal_alpha)
        ug, ugmin = _ug(uncertainty_gamma, uncertainty_gamma_min)
        norm = True if normalize_uncertainty is None else bool(normalize_uncertainty)
        kind = (label_loss or "sigmoid").lower()
        if kind not in {"sigmoid", "softmax"}:
            raise ValueError("label_loss must be either 'sigmoid' or 'softmax'")
        return ops.pairwise_mask_loss_forward(
            logits_for_kernels(mask_logits, mask_targets), mask_targets.contiguous(),
            cls_logits.contiguous().float(), cls_targets.contiguous(),
            smooth if smooth is not None else 1.0,
            sigmoid_scale if sigmoid_scale is not None else 1.0,
            dice_scale if dice_scale is not None else 1.0,
            cls_scale if cls_scale is not None else 1.0,
            background_index if background_index is not None else -1, ug, ugmin, mg, ma, cg, ca,
            kind == "softmax", norm)

    @staticmethod
    def backward(ctx, grad_output):
        return (None,) * 17


class PairwiseSigmoidCELossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, background_index, scale, focal_gamma, focal_alpha,
                uncertainty_gamma=None, uncertainty_gamma_min=None, normalize_uncertainty=True):
        assert logits.shape[1] == targets.shape[0], "Batch size mismatch between logits and targets"
        ug, ugmin = _ug(uncertainty_gamma, uncertainty_gamma_min)
        return ops.forward_pw_sigmoid_ce_loss(
            logits.contiguous().float(), targets.contiguous(),
            background_index if background_index is not None else -1,
            scale if scale is not None else 1.0, _gamma(focal_gamma), _alpha(focal_alpha), ug, ugmin,
            bool(normalize_uncertainty) if normalize_uncertainty is not None else True)

    @staticmethod
    def backward(ctx, grad_output):
        return (None,) * 9


class PairwiseDiceLossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, smooth, background_index, scale, uncertainty_gamma=None,
                uncertainty_gamma_min=None):
        assert logits.shape[1] == targets.shape[0], "Batch size mismatch between logits and targets"
        ug, ugmin = _ug(uncertainty_gamma, uncertainty_gamma_min)
        return ops.forward_pw_dice_loss(
            logits.contiguous().float(), targets.contiguous(), smooth if smooth is not None else 1.0,
            background_index if background_index is not None else -1,
            scale if scale is not None else 1.0, ug, ugmin)

    @staticmethod
    def backward(ctx, grad_output):
        return (None,) * 7


class PairwiseSigmoidLabelLossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, background_index=None, scale=1.0, focal_gamma=0.0,
                focal_alpha=None):
        return ops.forward_pw_sigmoid_label_loss(
            logits.contiguous().float(), targets.contiguous(),
            background_index if background_index is not None else -1,
            scale if scale is not None else 1.0, _gamma(focal_gamma), _alpha(focal_alpha))

    @staticmethod
    def backward(ctx, grad_output):
        return (None,) * 6


class PairwiseSoftmaxLabelLossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, background_index, scale):
        assert logits.shape[1] == targets.shape[0], "Batch size mismatch between logits and targets"
        return ops.forward_pw_softmax_label_loss(
            logits.contiguous().float(), targets.contiguous(),
            background_index if background_index is not None else -1,
            scale if scale is not None else 1.0)

    @staticmethod
    def backward(ctx, grad_output):
        return None, None, None, None


def pairwise_softmax_label_loss(logits, targets, background_index=None, scale=1.0):
    """functions/label/pw_softmax_label_loss.py:59-71."""
    return PairwiseSoftmaxLabelLossFunction.apply(logits, targets, background_index, scale)
