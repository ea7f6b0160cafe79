"""Autograd Functions with the names and signatures of the reference's
``functions`` package (functions/__init__.py:1-12 of AndyBarcia/mask_loss),
running on the B200 kernels of ``mask_loss_b200``.

The reference's pure-PyTorch ``*_py`` twins are its test oracles and are not
part of this package (the parity tests hold their own CPU oracle).
"""
from .matching import MaskMatchingFunction  # noqa: F401
from .pairwise import (  # noqa: F401
    PairwiseDiceLossFunction,
    PairwiseMaskLossFunction,
    PairwiseSigmoidCELossFunction,
    PairwiseSigmoidLabelLossFunction,
    PairwiseSoftmaxLabelLossFunction,
    pairwise_softmax_label_loss,
)
from .semantic import DiceLossFunction, SigmoidCELossFunction  # noqa: F401
from .sampled import (  # noqa: F401
    MaskMatchingSampledFunction,
    pairwise_dice_loss_sampling,
    pairwise_sigmoid_cross_entropy_loss_sampling,
)
from .losses import dice_loss, sigmoid_cross_entropy_loss  # noqa: F401
