"""Standalone semantic losses with the reference's Function signatures:
SigmoidCELossFunction (functions/sigmoid/sigmoid_ce.py:22-70) and
DiceLossFunction (functions/dice/dice_loss.py:14-50).  Per-layer losses of
(L,B,C,H,W) logits against a (B,H_t,W_t) label map; ``num_masks=None``
defaults to L*B*C as in the reference Functions."""
from torch.autograd import Function

from .. import ops


class SigmoidCELossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, num_masks, scale, focal_gamma=0.0, focal_alpha=None):
        L, B, C, h, w = logits.shape
        if B != targets.shape[0]:
            raise AssertionError("Batch size mismatch between logits and targets")
        ctx.num_masks = float(L * B * C) if num_masks is None else float(num_masks)
        ctx.scale = 1.0 if scale is None else float(scale)
        ctx.focal_gamma = 0.0 if focal_gamma is None else float(focal_gamma)
        if ctx.focal_gamma < 0.0:
            raise ValueError("focal_gamma must be non-negative")
        if focal_alpha is None:
            ctx.focal_alpha = -1.0
        else:
            ctx.focal_alpha = float(focal_alpha)
            if not 0.0 <= ctx.focal_alpha <= 1.0:
                raise ValueError("focal_alpha must be in [0, 1]")
        logits = logits.contiguous().float()
        targets = targets.contiguous()
        ctx.save_for_backward(logits, targets)
        return ops.forward_sigmoid_ce_loss(logits, targets, ctx.num_masks, ctx.scale,
                                           ctx.focal_gamma, ctx.focal_alpha)

    @staticmethod
    def backward(ctx, grad_output):
        logits, targets = ctx.saved_tensors
        g = ops.backward_sigmoid_ce_loss(grad_output.contiguous(), logits, targets, ctx.num_masks,
                                         ctx.scale, ctx.focal_gamma, ctx.focal_alpha)
        return g, None, None, None, None, None


class DiceLossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, smooth, num_masks, scale=1.0):
        L, B, C, h, w = logits.shape
        if B != targets.shape[0]:
            raise AssertionError("Batch size mismatch between logits and targets")
        ctx.num_masks = float(L * B * C) if num_masks is None else float(num_masks)
        ctx.scale = 1.0 if scale is None else float(scale)
        ctx.smooth = float(smooth)
        logits = logits.contiguous().float()
        targets = targets.contiguous().long()
        out, I, P, T = ops.forward_dice_loss(logits, targets, ctx.smooth, ctx.num_masks, ctx.scale)
        ctx.save_for_backward(logits, targets, I, P, T)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        logits, targets, I, P, T = ctx.saved_tensors
        g = ops.backward_dice_loss(grad_output.contiguous(), logits, targets, I, P, T, ctx.smooth,
                                   ctx.num_masks, ctx.scale)
        return g, None, None, None, None
