"""Full-size parity helpers: the CPU oracle run per image on host threads,
with the no-near-tie redraw filter of ``mask_loss_b200.synthetic``.

Images are independent in every cost, assignment and gradient (the reference
grids are (L,B,Q) / (Q,B,L), src/cuda/pw_mask.cu:408,
src/cuda/mask_matching_backward.cu:563; per-slice solve
src/cpu/matching.cpp:690-718), so the oracle's costs and mask gradients are
computed one image at a time, in parallel, and assembled.  Only the loss
denominators couple images (src/cuda/mask_matching_forward.cu:549-578): the
layer means are therefore taken by the oracle over the assembled batch, and
the per-image backward is given the batch's denominators (num_masks = the
batch's matched count when the call passes none; the class term's B*Q
denominator through a 1/B scale of the class upstream gradient).

Logits are drawn on the GPU with per-image generators (the values of an
image do not depend on which other images are drawn with it) and copied to
the host for the oracle.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from mask_loss_b200 import synthetic
from oracle import oracle as O

DEV = "cuda:0"
THREADS = max(1, min(32, os.cpu_count() or 1))


def _pool():
    return ThreadPoolExecutor(max_workers=THREADS)


class Case:
    """One full-size workload: GPU inputs, redraws and the oracle's results.

    cfg: a synthetic.Config (its L is the GPU call's layer count);
    images: the image indices to draw; layer: the layer the oracle checks
    (all layers when None); P: oracle Params of the call."""

    def __init__(self, cfg, images, P: O.Params, layer=None, eps=1e-4, log=print):
        self.cfg, self.images, self.P, self.layer = cfg, list(images), P, layer
        self._sep = {}
        self._host = {}

        def total(b, k):
            sep = self._image_sep(b, k)
            s32 = sep.astype(np.float32)
            t = ((s32[0] + s32[1]) + s32[2]).astype(np.float64)
            return t[0, 0]  # first checked layer, one image

        def solve(c):
            return O.assign_slice(c, P.inf_thresh, P.topk_matches, P.strategy_id)[0]

        # the expensive part of the filter (the oracle costs of k = 0) for
        # every image at once; redraws are rare and run one by one
        with _pool() as ex:
            list(ex.map(lambda b: self._image_sep(b, 0), self.images))
        self.redraws = synthetic.tie_free_redraws(
            cfg, self.images, total, solve, eps=eps,
            log=lambda b, k: log(f"{cfg.name} image {b}: {k} redraw(s)") if k else None)
        self.batch = synthetic.make_batch(cfg, images=self.images, device=DEV,
                                          redraws=self.redraws)
        self.Gmax = self.batch["cls_targets"].shape[1] - 1

    # -- per image ---------------------------------------------------------
    def _image_inputs(self, b, k):
        key = (b, k)
        if key not in self._host:
            one = synthetic.make_batch(self.cfg, images=[b], device=DEV, redraws={b: k})
            x = one["mask_logits"]
            z = one["cls_logits"]
            if self.layer is not None:
                x = x[self.layer:self.layer + 1]
                z = z[self.layer:self.layer + 1]
            self._host[key] = (x.float().cpu().numpy(), one["mask_targets"].cpu().numpy(),
                               z.cpu().numpy(), one["cls_targets"].cpu().numpy())
        return self._host[key]

    def _image_sep(self, b, k):
        key = (b, k)
        if key not in self._sep:
            x, t, z, y = self._image_inputs(b, k)
            self._sep[key] = O.pairwise_mask_loss(x, t, z, y, self.P)
        return self._sep[key]

    # -- assembled batch ---------------------------------------------------
    def oracle_costs(self) -> np.ndarray:
        """(3, Lc, B, Q, Gmax) costs; columns past an image's own GT count are
        +inf (no pixels, class -1), as the batch's padding makes them."""
        seps = [self._image_sep(b, self.redraws[b]) for b in self.images]
        Lc, Q = seps[0].shape[1], seps[0].shape[3]
        out = np.full((3, Lc, len(seps), Q, self.Gmax), np.inf)
        for i, s in enumerate(seps):
            out[:, :, i, :, :s.shape[4]] = s[:, :, 0]
        return out

    def oracle_forward(self):
        """pred_to_gt, pred_round, (3, Lc) means, costs."""
        sep = self.oracle_costs()
        s32 = sep.astype(np.float32)
        tot = (s32[0] + s32[1]) + s32[2]
        p2g, prd = O.match(tot, self.P)
        x = np.concatenate([self._image_inputs(b, self.redraws[b])[0] for b in self.images], 1)
        z = np.concatenate([self._image_inputs(b, self.redraws[b])[2] for b in self.images], 1)
        t = self.batch["mask_targets"].cpu().numpy()
        m, d, c = O.matched_loss_fwd(x, t, z, sep, p2g, self.P)
        return p2g, prd, np.stack([m, d, c]), sep

    def oracle_backward(self, p2g, gm, gd, gc):
        """Mask and class gradients of the checked layers, image by image."""
        P = self.P
        B = len(self.images)
        Lc = p2g.shape[0]
        matched = [(p2g[l] >= 0).sum() for l in range(Lc)]
        C = self._image_inputs(self.images[0], self.redraws[self.images[0]])[2].shape[3]
        has_void = 0 <= P.void_class_index < C
        cls_scale = (1.0 / B) if (P.force_unmatched_class_to_background or has_void) else 1.0
        gm, gd, gc = (np.asarray(v, np.float64).reshape(Lc) for v in (gm, gd, gc))

        def one(i):
            b = self.images[i]
            x, t, z, y = self._image_inputs(b, self.redraws[b])
            Pi = O.Params(**vars(P))
            if P.num_masks <= 0 and not P.force_unmatched_masks_to_empty:
                if Lc != 1:
                    raise ValueError("per-image backward with matched-count denominators "
                                     "needs one checked layer")
                Pi.num_masks = float(max(matched[0], 1))
            # image b's slice of the batch assignment, its own column count
            pg = p2g[:, i:i + 1].copy()
            pg[pg >= y.shape[1] - 1] = -1
            return O.mask_matching_backward(gm, gd, gc * cls_scale, x, t, z, y, pg, Pi)

        with _pool() as ex:
            res = list(ex.map(one, range(B)))
        return (np.concatenate([r[0] for r in res], 1), np.concatenate([r[1] for r in res], 1))
