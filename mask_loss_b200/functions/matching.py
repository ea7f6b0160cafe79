"""MaskMatchingFunction: the autograd bridge of functions/mask/matching.py:21-334.

Same 24 inputs in the same order, same defaulting and validation, same five
outputs.  Unlike the reference wrapper (which passes 25 positional arguments
to a 24-argument binding, functions/mask/matching.py:198-224) it calls the op
with the binding's own argument order.  The forward keeps the per-query
statistics of the matched pairs, so the backward streams the logits once.

``num_masks`` may also be a CUDA fp32 scalar tensor (for instance the result
of an all-reduce): it is then read on the device and never synchronised; or
the string ``"auto"``: the number of present non-background GT ids of the
batch, counted on the device from the forward's own label histogram.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from .. import ops

STRATEGIES = {"global": 0, "round": 1, "greedy": 2, "pseudo_greedy": 3}


def _f(v, default):
    return float(v if v is not None else default)


def resolve_args(mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale,
                 dice_scale, cls_scale, background_index, uncertainty_gamma,
                 uncertainty_gamma_min, normalize_uncertainty, inf_thresh, num_masks,
                 force_unmatched_class_to_background, force_unmatched_masks_to_empty, K,
                 assignment_strategy, mask_focal_gamma, mask_focal_alpha, cls_focal_gamma,
                 cls_focal_alpha, void_class_index=None, label_loss="sigmoid"):
    """Defaulting and validation of functions/mask/matching.py:104-196.
    Returns the binding's positional arguments after the four tensors, plus
    the device num_masks tensor (or None)."""
    if mask_logits.shape[1] != mask_targets.shape[0]:
        raise AssertionError("Batch size mismatch between logits and targets")
    ug = _f(uncertainty_gamma, 1.0)
    if ug < 0.0:
        raise ValueError("uncertainty_gamma must be non-negative")
    ugmin = _f(uncertainty_gamma_min, 0.05)
    if not 0.0 <= ugmin <= 1.0:
        raise ValueError("uncertainty_gamma_min must be in [0, 1]")
    norm = bool(normalize_uncertainty if normalize_uncertainty is not None else True)
    nm_dev = None
    if isinstance(num_masks, str) and num_masks == "auto":
        # count the present GT ids on the device during the forward; the count
        # lands in nm_dev and the backward reads it from there
        nm_dev = torch.empty((), dtype=torch.float32, device=mask_logits.device)
        nm = -2.0
    elif isinstance(num_masks, torch.Tensor):
        nm_dev = num_masks.detach().reshape(()).to(torch.float32).contiguous()
        nm = -1.0
    else:
        nm = _f(num_masks, -1.0)
    strategy = assignment_strategy if assignment_strategy is not None else "global"
    if strategy not in STRATEGIES:
        raise ValueError(f"Unknown assignment_strategy '{strategy}'."
                         f" Expected one of {sorted(STRATEGIES.keys())}")
    k = int(K if K is not None else 1)
    if k < 0:
        raise ValueError("K must be non-negative")
    mg = 0.0 if mask_focal_gamma is None else float(mask_focal_gamma)
    if mg < 0.0:
        raise ValueError("focal_gamma must be non-negative")
    if mask_focal_alpha is None:
        ma = -1.0
    else:
        ma = float(mask_focal_alpha)
        if not 0.0 <= ma <= 1.0:
            raise ValueError("focal_alpha must be in [0, 1]")
    if cls_focal_gamma is None:
        cg = mg
    else:
        cg = float(cls_focal_gamma)
        if cg < 0.0:
            raise ValueError("focal_gamma must be non-negative")
    if cls_focal_alpha is None:
        ca = ma
    else:
        ca = float(cls_focal_alpha)
        if not 0.0 <= ca <= 1.0:
            raise ValueError("focal_alpha must be in [0, 1]")
    C = cls_logits.shape[-1]
    if void_class_index is None:
        vi = -1
    else:
        vi = int(void_class_index)
        if not 0 <= vi < C:
            raise ValueError("incorrect void index")
    kind = (label_loss or "sigmoid").lower()
    if kind not in {"sigmoid", "softmax"}:
        raise ValueError("label_loss must be either 'sigmoid' or 'softmax'")
    softmax = kind == "softmax"
    force_cls = bool(force_unmatched_class_to_background or False)
    force_masks = bool(force_unmatched_masks_to_empty or False)
    if softmax and force_cls and vi == -1:
        raise ValueError("void_class_index must be provided when using softmax label loss "
                         "and forcing unmatched predictions to background")
    args = (_f(smooth, 1.0), _f(sigmoid_scale, 1.0), _f(dice_scale, 1.0), _f(cls_scale, 1.0),
            int(background_index if background_index is not None else -1), ug, ugmin,
            _f(inf_thresh, 1e30), nm, force_cls, force_masks, k, STRATEGIES[strategy], mg, ma, cg,
            ca, vi, softmax, norm)
    return args, nm_dev


def logits_for_kernels(mask_logits: torch.Tensor, mask_targets: torch.Tensor) -> torch.Tensor:
    """mask_logits as the kernels take them: bf16/fp16 kept, anything else
    fp32 (functions/mask/matching.py:109 upcasts always)."""
    x = mask_logits.contiguous()
    if x.dtype in (torch.bfloat16, torch.float16):
        return x
    return x.float()


class MaskMatchingFunction(Function):
    """Matching + matched losses; see functions/mask/matching.py:34-252."""

    @staticmethod
    def forward(ctx, mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale,
                dice_scale, cls_scale, background_index, uncertainty_gamma, uncertainty_gamma_min,
                normalize_uncertainty, inf_thresh, num_masks, force_unmatched_class_to_background,
                force_unmatched_masks_to_empty, K, assignment_strategy, mask_focal_gamma,
                mask_focal_alpha, cls_focal_gamma, cls_focal_alpha, void_class_index=None,
                label_loss="sigmoid"):
        # bf16/fp16 mask logits stay in their type (the kernels widen them;
        # the gradient comes back in the same type); anything else is upcast
        # as the reference does
        mask_logits = logits_for_kernels(mask_logits, mask_targets)
        mask_targets = mask_targets.contiguous()
        cls_logits = cls_logits.contiguous().float()
        cls_targets = cls_targets.contiguous()
        args, nm_dev = resolve_args(
            mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale, dice_scale,
            cls_scale, background_index, uncertainty_gamma, uncertainty_gamma_min,
            normalize_uncertainty, inf_thresh, num_masks, force_unmatched_class_to_background,
            force_unmatched_masks_to_empty, K, assignment_strategy, mask_focal_gamma,
            mask_focal_alpha, cls_focal_gamma, cls_focal_alpha, void_class_index, label_loss)
        # functions/mask/matching.py:180-181 (void id in cls_targets) is checked
        # on the device by the forward and raised without a host sync
        p2g, prd, means, saved, _ = ops.mask_matching_ex(
            mask_logits, mask_targets, cls_logits, cls_targets, *args,
            num_masks_dev=nm_dev, want_saved=True, check_void_targets=True)
        ctx.save_for_backward(mask_logits, mask_targets, cls_logits, cls_targets, p2g, saved,
                              nm_dev if nm_dev is not None else torch.empty(0))
        ctx.args = args
        ctx.has_nm_dev = nm_dev is not None
        ctx.mark_non_differentiable(p2g, prd)
        return p2g, prd, means[0], means[1], means[2]

    @staticmethod
    def backward(ctx, _g0, _g1, grad_mask_mean, grad_dice_mean, grad_cls_mean):
        ml, mt, cl, ct, p2g, saved, nm_dev = ctx.saved_tensors
        a = ctx.args
        L = ml.shape[0]

        def g(x):
            if x is None:
                return torch.zeros(L, dtype=torch.float32, device=ml.device)
            return x.contiguous().float()

        gm, gc = ops.mask_matching_backward(
            g(grad_mask_mean), g(grad_dice_mean), g(grad_cls_mean), ml, mt, cl, ct, p2g,
            a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[8], a[9], a[10], a[13], a[14], a[15], a[16],
            a[17], a[18], a[19], saved=saved,
            num_masks_dev=nm_dev if ctx.has_nm_dev else None)
        return (gm, None, gc) + (None,) * 21
