"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No dataset is involved: every tensor is drawn from a seeded generator with the
shapes, sizes and value distributions of the configurations below.  GT masks
are painted into a label map in id order, so later masks occlude earlier ones
(the reference API takes label maps, src/bindings.cpp:66); a GT that ends up
fully occluded becomes an absent column (+inf cost), exactly as in the
reference.  Column 0 is background (``background_index=0``), ``cls_targets``
is (B, max_b G_b + 1) with -1 padding, classes drawn from the real classes
[0, C'-1) so the void class C'-1 never appears as a target.

Per-image seeds are ``1000 * cfg + b`` so a subset of images can be
regenerated independently (the CPU baseline uses that).  A redrawn image
(``redraws={b: k}``) adds ``10**6 * k`` to each of its seeds.

No-near-tie filter (``tie_free_redraws``): an image is kept only when its
assignment survives a relative perturbation of its total costs,
``cost * (1 + eps * U[-1, 1])``; otherwise it is redrawn with the next k.
The caller supplies the costs and the solver (the library itself has no CPU
arithmetic), so the filter is run by the parity tests with their checker.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class Config:
    name: str
    cfg: int
    L: int
    B: int
    Q: int
    H: int
    W: int
    s: int            # label map is (H*s, W*s)
    C: int            # classes + 1 (void = C-1)
    logit_std: float
    shapes: str       # "ellipse", "ellipse_rect", "polygon", "video"
    g_law: tuple      # ("fixed", n) | ("poisson", lam, lo, hi) | ("uniform", lo, hi)
    area: tuple       # area fraction range
    frames: int = 1   # video: frames stacked vertically (H = frames * frame_h)


CONFIGS = {
    "cfg1": Config("cfg1", 1, 1, 2, 100, 64, 64, 1, 81, 3.0, "ellipse", ("fixed", 8), (0.005, 0.30)),
    "cfg2": Config("cfg2", 2, 1, 16, 100, 256, 256, 1, 134, 3.0, "ellipse_rect",
                   ("poisson", 15, 1, 100), (0.001, 0.40)),
    "cfg4": Config("cfg4", 4, 1, 64, 200, 512, 512, 1, 151, 4.0, "polygon", ("uniform", 20, 200),
                   (0.0005, 0.20)),
    "cfg5": Config("cfg5", 5, 1, 8, 200, 640, 128, 1, 41, 3.0, "video", ("uniform", 1, 30),
                   (0.002, 0.10), frames=5),
    "cfg3": Config("cfg3", 3, 1, 16, 100, 128, 128, 4, 134, 3.0, "ellipse_rect",
                   ("poisson", 15, 1, 100), (0.001, 0.40)),
    "native": Config("native", 6, 1, 8, 128, 256, 256, 4, 128, 1.0, "ellipse", ("uniform", 10, 19),
                     (0.002, 0.05)),
}

CFG3_POINTS = 12544  # points per image of the point-sampled configuration (112 x 112)


# Matching/loss arguments of the parity settings: softmax label loss over C'
# classes with void = C'-1, unmatched queries pushed to void, K=1 global
# Hungarian, weights class 2, sigmoid-CE 5, dice 5.
def parity_kwargs(cfg: Config, uncertainty_gamma: float = 0.0) -> dict:
    return dict(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
                uncertainty_gamma=uncertainty_gamma, uncertainty_gamma_min=0.05, inf_thresh=1e30,
                num_masks=-1.0, force_unmatched_class_to_background=True,
                force_unmatched_masks_to_empty=False, topk_matches=1, strategy_id=0,
                mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0, cls_alpha=-1.0,
                void_class_index=cfg.C - 1, use_softmax_label_loss=True,
                normalize_uncertainty=True)


def _n_gt(law, rng) -> int:
    if law[0] == "fixed":
        return int(law[1])
    if law[0] == "poisson":
        return int(min(max(rng.poisson(law[1]), law[2]), law[3]))
    return int(rng.integers(law[1], law[2] + 1))


def _paint_ellipse(lab, gid, cy, cx, ry, rx, rng_theta=0.0):
    Ht, Wt = lab.shape
    y0, y1 = max(0, int(cy - ry - 1)), min(Ht, int(cy + ry + 2))
    x0, x1 = max(0, int(cx - rx - 1)), min(Wt, int(cx + rx + 2))
    if y0 >= y1 or x0 >= x1:
        return
    yy, xx = np.mgrid[y0:y1, x0:x1]
    m = ((yy + 0.5 - cy) / max(ry, 0.5)) ** 2 + ((xx + 0.5 - cx) / max(rx, 0.5)) ** 2 <= 1.0
    lab[y0:y1, x0:x1][m] = gid


def _paint_rect(lab, gid, cy, cx, hy, hx):
    Ht, Wt = lab.shape
    y0, y1 = max(0, int(round(cy - hy))), min(Ht, int(round(cy + hy)) + 1)
    x0, x1 = max(0, int(round(cx - hx))), min(Wt, int(round(cx + hx)) + 1)
    if y0 < y1 and x0 < x1:
        lab[y0:y1, x0:x1] = gid


def _paint_polygon(lab, gid, cy, cx, r, nv, rng):
    Ht, Wt = lab.shape
    ang = np.sort(rng.uniform(0, 2 * math.pi, nv))
    rad = r * rng.uniform(0.6, 1.4, nv)
    py = cy + rad * np.sin(ang)
    px = cx + rad * np.cos(ang)
    y0, y1 = max(0, int(py.min()) - 1), min(Ht, int(py.max()) + 2)
    x0, x1 = max(0, int(px.min()) - 1), min(Wt, int(px.max()) + 2)
    if y0 >= y1 or x0 >= x1:
        return
    yy, xx = np.mgrid[y0:y1, x0:x1]
    yy = yy + 0.5
    xx = xx + 0.5
    inside = np.zeros(yy.shape, bool)
    j = nv - 1
    for i in range(nv):  # even-odd rule
        yi, xi, yj, xj = py[i], px[i], py[j], px[j]
        cond = ((yi > yy) != (yj > yy)) & (xx < (xj - xi) * (yy - yi) / (yj - yi + 1e-12) + xi)
        inside ^= cond
        j = i
    lab[y0:y1, x0:x1][inside] = gid


REDRAW_SEED_STEP = 10 ** 6


def make_image_labels(cfg: Config, b: int, redraw: int = 0):
    """(H*s, W*s) int64 label map and the number of GT ids painted for image b."""
    rng = np.random.default_rng(1000 * cfg.cfg + b + REDRAW_SEED_STEP * redraw)
    Ht, Wt = cfg.H * cfg.s, cfg.W * cfg.s
    G = _n_gt(cfg.g_law, rng)
    lab = np.zeros((Ht, Wt), np.int64)
    if cfg.shapes == "video":
        fh = Ht // cfg.frames
        for gid in range(1, G + 1):
            a = rng.uniform(*cfg.area) * fh * Wt
            ry = math.sqrt(a / math.pi) * rng.uniform(0.7, 1.4)
            rx = a / (math.pi * ry)
            cy, cx = rng.uniform(0, fh), rng.uniform(0, Wt)
            for f in range(cfg.frames):
                cy_f = cy + rng.normal(0, 4.0) * f
                cx_f = cx + rng.normal(0, 4.0) * f
                sub = lab[f * fh:(f + 1) * fh]
                _paint_ellipse(sub, gid, cy_f, cx_f, ry, rx)
        return lab, G
    for gid in range(1, G + 1):
        a = rng.uniform(*cfg.area) * Ht * Wt
        cy, cx = rng.uniform(0, Ht), rng.uniform(0, Wt)
        kind = cfg.shapes
        if kind == "ellipse_rect":
            kind = "ellipse" if rng.random() < 0.5 else "rect"
        if kind == "ellipse":
            ry = math.sqrt(a / math.pi) * rng.uniform(0.6, 1.6)
            rx = a / (math.pi * ry)
            _paint_ellipse(lab, gid, cy, cx, ry, rx)
        elif kind == "rect":
            hy = math.sqrt(a) / 2 * rng.uniform(0.6, 1.6)
            hx = a / (4 * hy)
            _paint_rect(lab, gid, cy, cx, hy, hx)
        else:
            _paint_polygon(lab, gid, cy, cx, math.sqrt(a / math.pi), int(rng.integers(5, 13)), rng)
    return lab, G


def make_batch(cfg: Config, images=None, device="cpu", logits=True, redraws=None):
    """Inputs of one step: mask_logits (L,B,Q,H,W) f32, mask_targets (B,Ht,Wt)
    i64, cls_logits (L,B,Q,C) f32, cls_targets (B,GTmax+1) i64.

    `images` selects a subset of image indices (default: all B); `redraws`
    maps an image index to its redraw count k (default 0)."""
    idx = list(range(cfg.B)) if images is None else list(images)
    rd = {} if redraws is None else dict(redraws)
    ks = [int(rd.get(b, 0)) for b in idx]
    labs, gs = zip(*(make_image_labels(cfg, b, k) for b, k in zip(idx, ks)))
    gmax = max(gs)
    cls = np.full((len(idx), gmax + 1), -1, np.int64)
    for i, b in enumerate(idx):
        rng = np.random.default_rng(10_000_000 + 1000 * cfg.cfg + b + REDRAW_SEED_STEP * ks[i])
        cls[i, 1:gs[i] + 1] = rng.integers(0, cfg.C - 1, gs[i])
    targets = torch.from_numpy(np.stack(labs)).to(device)
    cls_t = torch.from_numpy(cls).to(device)
    out = {"mask_targets": targets, "cls_targets": cls_t}
    if logits:
        # one generator per image, so any subset of images gets the same values
        ml, cl = [], []
        for b, k in zip(idx, ks):
            seed = 1000 * cfg.cfg + 7 + 100003 * b + REDRAW_SEED_STEP * k
            if str(device).startswith("cuda"):
                g = torch.Generator(device=device).manual_seed(seed)
            else:
                g = torch.Generator().manual_seed(seed)
            ml.append(torch.randn((cfg.L, 1, cfg.Q, cfg.H, cfg.W), generator=g, device=device))
            cl.append(torch.randn((cfg.L, 1, cfg.Q, cfg.C), generator=g, device=device))
        out["mask_logits"] = torch.cat(ml, 1) * cfg.logit_std
        out["cls_logits"] = torch.cat(cl, 1)
    return out


def tie_free_redraws(cfg: Config, images, total_cost, solve, eps: float = 1e-4,
                     max_redraws: int = 32, log=None) -> dict:
    """Redraw counts {b: k} that make every listed image free of near-ties.

    For image b and k = 0, 1, ...: ``total_cost(b, k)`` returns its (Q, G)
    float64 total cost matrix and ``solve(cost)`` its assignment (an int
    array).  The draw is kept when the assignment of
    ``cost * (1 + eps * U[-1, 1])`` (U seeded by b and k) equals that of
    ``cost``.  eps defaults to the 1e-4 relative cost tolerance of the
    parity contract: an assignment that a perturbation of that size can
    change is a tie under that contract.  `log(b, k)` is called with the
    final k of each image."""
    out = {}
    for b in images:
        for k in range(max_redraws + 1):
            c = np.asarray(total_cost(b, k), np.float64)
            rng = np.random.default_rng(7_000_000 + 1000 * cfg.cfg + b + REDRAW_SEED_STEP * k)
            pert = c * (1.0 + eps * rng.uniform(-1.0, 1.0, c.shape))
            pert[~np.isfinite(c)] = c[~np.isfinite(c)]
            if np.array_equal(np.asarray(solve(c)), np.asarray(solve(pert))):
                out[b] = k
                break
        else:
            raise RuntimeError(f"image {b}: no tie-free draw in {max_redraws} redraws")
        if log is not None:
            log(b, out[b])
    return out
