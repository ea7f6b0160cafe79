"""Point-sampled costs and matching (config 3).

``pairwise_sigmoid_cross_entropy_loss_sampling`` / ``pairwise_dice_loss_sampling``
are the GPU counterparts of the reference's
pairwise_sigmoid_cross_entropy_loss_sampling_py (functions/sigmoid/pw_sigmoid_ce.py:407-549)
and pairwise_dice_loss_sampling_py (functions/dice/pw_dice_loss.py:174-268):
same arguments, same point draws (``torch.rand(1,P,2)`` per image with a
non-background GT id, on the logits' device) unless ``point_coords`` is given.

``MaskMatchingSampledFunction`` matches and computes the matched losses and
gradients on those point costs.  The reference has no such op (it never
wires sampling into matching, functions/mask/matching.py:836); its semantics
follow MaskMatchingFunction with the point costs in place of the dense ones.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from .. import ops
from .matching import STRATEGIES


def _bg(background_index):
    return -1 if background_index is None else int(background_index)


def _sampled_costs(logits, targets, background_index, num_points, align_corners, point_coords,
                   which, smooth=1.0, scale=1.0, focal_gamma=0.0, focal_alpha=None, num_gts=None):
    bg = _bg(background_index)
    # GT_total sets the output's width: read from the targets on the host
    # unless the caller passes it (num_gts)
    if num_gts is not None:
        gt_total = int(num_gts)
    else:
        gt_total = int(targets.max().item()) + 1 if targets.numel() else 0
    L, B, Q = logits.shape[:3]
    if point_coords is None:
        point_coords = ops.reference_point_coords(targets, num_points, bg)
    cls_logits = torch.zeros((L, B, Q, 1), dtype=torch.float32, device=logits.device)
    cls_targets = torch.full((B, max(gt_total, 0)), -1, dtype=torch.int64, device=logits.device)
    out = ops.pairwise_mask_loss_sampled_forward(
        logits.contiguous(), targets.contiguous(), cls_logits, cls_targets,
        point_coords.contiguous().float(), smooth, scale, scale, 1.0, bg,
        float(focal_gamma or 0.0), -1.0 if focal_alpha is None else float(focal_alpha), 0.0, -1.0,
        False, align_corners)
    return out if out.dim() == 4 else out[which].contiguous()


def pairwise_sigmoid_cross_entropy_loss_sampling(logits, targets, background_index=None, scale=1.0,
                                                 num_points=5000, align_corners=False,
                                                 focal_gamma=0.0, focal_alpha=None,
                                                 point_coords=None, *, num_gts=None):
    """num_gts (keyword): targets.max() + 1 when known, to skip the host read."""
    return _sampled_costs(logits, targets, background_index, num_points, align_corners,
                          point_coords, 0, scale=scale, focal_gamma=focal_gamma,
                          focal_alpha=focal_alpha, num_gts=num_gts)


def pairwise_dice_loss_sampling(logits, targets, smooth=1.0, background_index=None, scale=1.0,
                                num_points=5000, align_corners=False, point_coords=None, *,
                                num_gts=None):
    """num_gts (keyword): targets.max() + 1 when known, to skip the host read."""
    return _sampled_costs(logits, targets, background_index, num_points, align_corners,
                          point_coords, 1, smooth=smooth, scale=scale, num_gts=num_gts)


def resolve_sampled_args(smooth, sigmoid_scale, dice_scale, cls_scale, background_index, inf_thresh,
                         num_masks, force_unmatched_class_to_background, K, assignment_strategy,
                         mask_focal_gamma, mask_focal_alpha, cls_focal_gamma, cls_focal_alpha,
                         void_class_index=None, label_loss="sigmoid", align_corners=False,
                         device=None):
    """Defaulting and validation of the sampled Function's scalar arguments.
    Returns the op's positional arguments and the device num_masks (or None).
    ``num_masks="auto"``: the present non-background GT ids of the batch,
    counted on ``device`` by the forward from its full-resolution label
    histogram."""
    if assignment_strategy not in STRATEGIES:
        raise ValueError(f"Unknown assignment_strategy '{assignment_strategy}'.")
    softmax = (label_loss or "sigmoid").lower() == "softmax"
    vi = -1 if void_class_index is None else int(void_class_index)
    if softmax and force_unmatched_class_to_background and vi == -1:
        raise ValueError("void_class_index must be provided when using softmax label loss "
                         "and forcing unmatched predictions to background")
    mg = float(mask_focal_gamma or 0.0)
    ma = -1.0 if mask_focal_alpha is None else float(mask_focal_alpha)
    cg = mg if cls_focal_gamma is None else float(cls_focal_gamma)
    ca = ma if cls_focal_alpha is None else float(cls_focal_alpha)
    nm_dev = None
    nm = -1.0
    if isinstance(num_masks, str) and num_masks == "auto":
        nm_dev = torch.empty((), dtype=torch.float32, device=device)
        nm = -2.0
    elif isinstance(num_masks, torch.Tensor):
        nm_dev = num_masks.detach().reshape(()).to(torch.float32).contiguous()
    elif num_masks is not None:
        nm = float(num_masks)
    args = (float(smooth), float(sigmoid_scale), float(dice_scale), float(cls_scale),
            _bg(background_index), float(inf_thresh), nm,
            bool(force_unmatched_class_to_background), int(K), STRATEGIES[assignment_strategy],
            mg, ma, cg, ca, vi, softmax, bool(align_corners))
    return args, nm_dev


class MaskMatchingSampledFunction(Function):
    """Inputs: mask_logits (L,B,Q,H,W) fp32/bf16, mask_targets, cls_logits,
    cls_targets, point_coords (B,P,2) in [0,1], then smooth, sigmoid_scale,
    dice_scale, cls_scale, background_index, inf_thresh, num_masks (float,
    None or CUDA scalar), force_unmatched_class_to_background, K,
    assignment_strategy, mask_focal_gamma, mask_focal_alpha, cls_focal_gamma,
    cls_focal_alpha, void_class_index=None, label_loss="sigmoid",
    align_corners=False.  Outputs as MaskMatchingFunction."""

    @staticmethod
    def forward(ctx, mask_logits, mask_targets, cls_logits, cls_targets, point_coords, smooth,
                sigmoid_scale, dice_scale, cls_scale, background_index, inf_thresh, num_masks,
                force_unmatched_class_to_background, K, assignment_strategy, mask_focal_gamma,
                mask_focal_alpha, cls_focal_gamma, cls_focal_alpha, void_class_index=None,
                label_loss="sigmoid", align_corners=False):
        args, nm_dev = resolve_sampled_args(
            smooth, sigmoid_scale, dice_scale, cls_scale, background_index, inf_thresh, num_masks,
            force_unmatched_class_to_background, K, assignment_strategy, mask_focal_gamma,
            mask_focal_alpha, cls_focal_gamma, cls_focal_alpha, void_class_index, label_loss,
            align_corners, device=mask_logits.device)
        ml = mask_logits.contiguous()
        cl = cls_logits.contiguous().float()
        pc = point_coords.contiguous().float()
        p2g, prd, means, saved, _, fws = ops.mask_matching_sampled_ex(
            ml, mask_targets.contiguous(), cl, cls_targets.contiguous(), pc, *args,
            num_masks_dev=nm_dev, want_saved=True, want_workspace=True)
        ctx.save_for_backward(ml, mask_targets, cl, cls_targets, pc, p2g, saved,
                              nm_dev if nm_dev is not None else torch.empty(0), fws)
        ctx.args = args
        ctx.has_nm = nm_dev is not None
        ctx.mark_non_differentiable(p2g, prd)
        return p2g, prd, means[0], means[1], means[2]

    @staticmethod
    def backward(ctx, _a, _b, gm_mean, gd_mean, gc_mean):
        ml, mt, cl, ct, pc, p2g, saved, nm_dev, fws = ctx.saved_tensors
        a = ctx.args
        L = ml.shape[0]

        def g(x):
            return (torch.zeros(L, dtype=torch.float32, device=ml.device) if x is None
                    else x.contiguous().float())

        gm, gc = ops.mask_matching_sampled_backward(
            g(gm_mean), g(gd_mean), g(gc_mean), ml, mt, cl, ct, pc, p2g, saved, a[0], a[1], a[2],
            a[3], a[4], a[6], a[7], a[10], a[11], a[12], a[13], a[14], a[15], a[16],
            num_masks_dev=nm_dev if ctx.has_nm else None, forward_workspace=fws)
        return (gm, None, gc) + (None,) * 19
