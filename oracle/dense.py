"""CPU oracle of the dense per-GT mask target mode.

TEST INFRASTRUCTURE ONLY (tests/); the product never imports it.

The reference has no dense-mask mode (its API takes a label map,
src/bindings.cpp:66).  This oracle defines it through the pinned label-map
oracle (oracle.py): the costs of GT column g depend only on which pixels
carry g's label, so column g is the label-map cost of a map that holds g's id
on g's mask and an ignored id (-1) elsewhere; a prediction's gradient uses
only its matched GT's mask, so its row comes from the label-map backward with
that GT's map.  On non-overlapping masks this equals the label-map oracle of
the combined map.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def _gout_cols(GT_total: int, bg: int):
    return [k for k in range(GT_total) if not (0 <= bg < GT_total and k == bg)]


def _map_for(masks, ga):
    m = np.asarray(masks)
    t = np.full((m.shape[0],) + m.shape[2:], -1, np.int64)
    t[m[:, ga] != 0] = ga
    return t


def pairwise_costs(mask_logits, masks, cls_logits, cls_targets, P: O.Params):
    """(3,L,B,Q,GT_out) costs against dense masks (B,GT_total,Ht,Wt)."""
    GT_total = np.asarray(cls_targets).shape[1]
    cols = _gout_cols(GT_total, P.background_index)
    out = None
    for g, ga in enumerate(cols):
        sep = O.pairwise_mask_loss(mask_logits, _map_for(masks, ga), cls_logits, cls_targets, P)
        if out is None:
            out = np.empty_like(sep)
        out[..., g] = sep[..., g]
    return out


def mask_matching(mask_logits, masks, cls_logits, cls_targets, P: O.Params):
    """pred_to_gt, pred_round, mask/dice/class layer means, (3,...) costs."""
    sep = pairwise_costs(mask_logits, masks, cls_logits, cls_targets, P)
    sep32 = sep.astype(np.float32)
    total = (sep32[0] + sep32[1]) + sep32[2]
    p2g, prd = O.match(total, P)
    m, d, c = O.matched_loss_fwd(mask_logits, _map_for(masks, 0), cls_logits, sep, p2g, P)
    return p2g, prd, m, d, c, sep


def mask_matching_backward(gm, gd, gc, mask_logits, masks, cls_logits, cls_targets, p2g,
                           P: O.Params):
    """(grad_mask_logits, grad_cls_logits)."""
    GT_total = np.asarray(cls_targets).shape[1]
    cols = _gout_cols(GT_total, P.background_index)
    p2g = np.asarray(p2g)
    gx, gz = O.mask_matching_backward(gm, gd, gc, mask_logits, _map_for(masks, cols[0] if cols else 0),
                                      cls_logits, cls_targets, p2g, P)
    gx = gx.copy()
    for g, ga in enumerate(cols):
        rows = p2g == g
        if not rows.any():
            continue
        gxg, _ = O.mask_matching_backward(gm, gd, gc, mask_logits, _map_for(masks, ga), cls_logits,
                                          cls_targets, p2g, P)
        gx[rows] = gxg[rows]
    return gx, gz
