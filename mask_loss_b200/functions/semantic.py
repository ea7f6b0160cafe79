"""Standalone semantic losses (functions/sigmoid/sigmoid_ce.py:22-70,
functions/dice/dice_loss.py:14-50).  They are not on the matching path and
are not implemented in this build; using them raises NotImplementedError."""
from torch.autograd import Function


class SigmoidCELossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, num_masks, scale, focal_gamma=0.0, focal_alpha=None):
        raise NotImplementedError("SigmoidCELossFunction is not implemented in mask_loss_b200")


class DiceLossFunction(Function):
    @staticmethod
    def forward(ctx, logits, targets, smooth, num_masks, scale=1.0):
        raise NotImplementedError("DiceLossFunction is not implemented in mask_loss_b200")
