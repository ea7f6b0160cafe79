"""Golden fixtures of the standalone semantic losses, made by the reference.

    python tests/golden/make_golden_semantic.py      (needs the reference checkout: MASK_LOSS_REF)

``semantic_*.npz``: inputs, the per-layer losses of the reference's
``sigmoid_cross_entropy_loss_py`` (functions/sigmoid/sigmoid_ce.py:147-226) and
``dice_loss_py`` (functions/dice/dice_loss.py:100-168) in float64, and the
autograd gradients of ``sum_l g_l * loss_l``.  Tests read only the .npz files.
"""
import contextlib
import io
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.oracle import reference_root  # noqa: E402

REF = reference_root()
if REF is None:
    raise SystemExit("reference checkout not found: set MASK_LOSS_REF")
sys.path.insert(0, REF)
with contextlib.redirect_stdout(io.StringIO()):
    import functions as RF  # noqa: E402  (the reference's Python package)

# name: (L, B, C, H, W, s, seed, sigmoid kwargs, dice kwargs)
CASES = {
    "semantic_s1": (2, 2, 5, 6, 7, 1, 1, dict(num_masks=7.0, scale=1.5),
                    dict(smooth=1.0, num_masks=5.0, scale=2.0)),
    "semantic_s2_focal": (1, 3, 4, 5, 5, 2, 2,
                          dict(num_masks=3.0, scale=1.0, focal_gamma=2.0, focal_alpha=0.25),
                          dict(smooth=0.5, num_masks=12.0, scale=1.0)),
    "semantic_s4_gamma": (2, 1, 6, 4, 3, 4, 3, dict(num_masks=2.0, scale=0.7, focal_gamma=1.5),
                          dict(smooth=1e-6, num_masks=6.0, scale=1.3)),
}


def main():
    for name, (L, B, C, H, W, s, seed, skw, dkw) in CASES.items():
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(L, B, C, H, W, generator=g, dtype=torch.float32) * 3.0).double()
        # blocky label maps, so pure and mixed cells both occur
        lab = torch.randint(0, C, (B, H * s // max(1, s // 2), W * s // max(1, s // 2)), generator=g)
        lab = lab.repeat_interleave(max(1, s // 2), 1).repeat_interleave(max(1, s // 2), 2)
        t = lab[:, :H * s, :W * s].contiguous()
        go = torch.rand(L, generator=g, dtype=torch.float64) + 0.5
        xs = x.clone().requires_grad_(True)
        ls = RF.sigmoid_cross_entropy_loss_py(xs, t, **skw)
        (ls * go).sum().backward()
        xd = x.clone().requires_grad_(True)
        ld = RF.dice_loss_py(xd, t, **dkw)
        (ld * go).sum().backward()
        np.savez(os.path.join(HERE, name + ".npz"), logits=x.float().numpy(), targets=t.numpy(),
                 grad_out=go.numpy(), sce_loss=ls.detach().numpy(), sce_grad=xs.grad.numpy(),
                 dice_loss=ld.detach().numpy(), dice_grad=xd.grad.numpy(),
                 sce_kw=np.array([skw["num_masks"], skw["scale"], skw.get("focal_gamma", 0.0),
                                  skw.get("focal_alpha", -1.0)]),
                 dice_kw=np.array([dkw["smooth"], dkw["num_masks"], dkw["scale"]]))
        print(name, ls.detach().numpy(), ld.detach().numpy())


if __name__ == "__main__":
    main()
