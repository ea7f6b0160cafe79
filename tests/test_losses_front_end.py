"""Argument handling of the functions/losses.py front-end (no GPU needed:
every case raises before a kernel would run)."""
import pytest
import torch

from mask_loss_b200 import functions as F


@pytest.mark.parametrize("fn", [F.sigmoid_cross_entropy_loss, F.dice_loss])
def test_rejects_what_it_does_not_provide(fn):
    x = torch.zeros(2, 3, 4, 4)
    t = torch.zeros(2, 4, 4, dtype=torch.int64)
    with pytest.raises(ValueError, match="class_mapping"):
        fn(x, t, class_mapping=torch.arange(256))
    with pytest.raises(ValueError, match="CUDA only"):
        fn(x, t, implementation="python")
    with pytest.raises(ValueError, match="logits must be"):
        fn(torch.zeros(3, 4, 4), t)
