"""Time the reference's own pure-PyTorch path on the host CPU.

TEST INFRASTRUCTURE ONLY (a measurement, nothing of the product runs here).

    MASK_LOSS_REF=<reference checkout> python oracle/time_reference_py.py [cfg2] [images]

``mask_matching_py`` (functions/mask/matching.py:336-815 of the reference:
pairwise costs, scipy assignment, matched losses) forward plus its autograd
backward, on seeded synthetic images of a configuration of
mask_loss_b200/synthetic.py (the parity settings), one image per call, with
``torch.set_num_threads(os.cpu_count())``.  Prints images/s and the thread
count.  The reference's Python package cannot be shipped to the GPU box, so
this runs where the checkout is.
"""
from __future__ import annotations

import contextlib
import io
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:] = [q for q in sys.path if os.path.abspath(q or ".") != HERE]
sys.path.insert(0, os.path.dirname(HERE))

import torch  # noqa: E402

from mask_loss_b200 import synthetic  # noqa: E402
from oracle.oracle import reference_root  # noqa: E402


def main():
    root = reference_root()
    if root is None:
        raise SystemExit("reference checkout not found: set MASK_LOSS_REF")
    sys.path.insert(0, root)
    with contextlib.redirect_stdout(io.StringIO()):
        from functions.mask.matching import mask_matching_py
    name = sys.argv[1] if len(sys.argv) > 1 else "cfg2"
    n = int(sys.argv[2]) if len(sys.argv) > 2 else 4
    cfg = synthetic.CONFIGS[name]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    kw = synthetic.parity_kwargs(cfg)
    total = 0.0
    for b in range(n):
        bt = synthetic.make_batch(cfg, images=[b])
        x = bt["mask_logits"].clone().requires_grad_(True)
        z = bt["cls_logits"].clone().requires_grad_(True)
        t0 = time.perf_counter()
        out = mask_matching_py(x, bt["mask_targets"], z, bt["cls_targets"], kw["smooth"],
                               kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
                               kw["background_index"], kw["uncertainty_gamma"],
                               kw["uncertainty_gamma_min"], True, kw["inf_thresh"], None,
                               kw["force_unmatched_class_to_background"],
                               kw["force_unmatched_masks_to_empty"], 1, "global", 0.0, None, None,
                               None, kw["void_class_index"], "softmax")
        (out[2] + out[3] + out[4]).sum().backward()
        total += time.perf_counter() - t0
    print(f"mask_matching_py fwd+bwd, {name}, {n} images one per call, {threads} threads: "
          f"{n / total:.2f} images/s ({total / n * 1e3:.0f} ms per image)")


if __name__ == "__main__":
    main()
