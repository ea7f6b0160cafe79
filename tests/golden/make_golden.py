"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference checkout exists (MASK_LOSS_REF, or a ``reference``
directory beside the repository):

    python tests/golden/make_golden.py

* ``mm_*.npz``: inputs and outputs of the reference's pure-PyTorch path
  ``functions.mask.matching.mask_matching_py`` (functions/mask/matching.py:336-815)
  and ``functions.mask.pw_mask.pairwise_mask_loss_py`` (functions/mask/pw_mask.py:118-186),
  evaluated in float64 on float32-representable inputs, plus the autograd
  gradients of ``sum_l a_l*mask_mean + b_l*dice_mean + c_l*cls_mean``.
* ``solver.npz``: fp64 cost slices and the assignments that the reference's
  C++ solver (src/cpu/matching.cpp:476-571, compiled by oracle/Makefile into
  oracle/_ref/libref.so) returns for strategies 0-3 and K in {0,1,2,3}.

Fixtures are small (a few hundred KB total).  Nothing of the reference is
read at test time: the tests only read these .npz files.
"""
import contextlib
import io
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.oracle import reference_root  # noqa: E402

REF = reference_root()
if REF is None:
    raise SystemExit("reference checkout not found: set MASK_LOSS_REF")
sys.path.insert(0, REPO)
sys.path.insert(0, REF)

with contextlib.redirect_stdout(io.StringIO()):
    import functions as RF  # noqa: E402  (the reference's Python package)
from oracle import oracle as O  # noqa: E402

STRATS = ["global", "round", "greedy", "pseudo_greedy"]

# name: (L,B,Q,H,W,s,C,G, kwargs)
CASES = {
    "mm_parity_softmax": (2, 2, 12, 8, 8, 1, 7, 5, dict(
        smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
        uncertainty_gamma=0.0, uncertainty_gamma_min=0.05, num_masks=None,
        force_unmatched_class_to_background=True, force_unmatched_masks_to_empty=False,
        K=1, assignment_strategy="global", void_class_index=6, label_loss="softmax")),
    "mm_uncert_sigmoid_focal": (1, 3, 10, 6, 10, 1, 5, 4, dict(
        smooth=1.0, sigmoid_scale=2.0, dice_scale=3.0, cls_scale=1.5, background_index=0,
        uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, num_masks=4.0,
        force_unmatched_class_to_background=False, force_unmatched_masks_to_empty=False,
        K=1, assignment_strategy="global", mask_focal_gamma=2.0, mask_focal_alpha=0.25,
        cls_focal_gamma=1.5, cls_focal_alpha=0.3, label_loss="sigmoid")),
    "mm_s2_forced_k2": (1, 2, 14, 6, 6, 2, 6, 4, dict(
        smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
        uncertainty_gamma=0.0, uncertainty_gamma_min=0.05, num_masks=None,
        force_unmatched_class_to_background=True, force_unmatched_masks_to_empty=True,
        K=2, assignment_strategy="global", void_class_index=5, label_loss="softmax")),
    "mm_round_k2_nobg": (2, 2, 9, 5, 7, 1, 4, 3, dict(
        smooth=0.5, sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0, background_index=-1,
        uncertainty_gamma=1.0, uncertainty_gamma_min=0.1, num_masks=None,
        force_unmatched_class_to_background=True, force_unmatched_masks_to_empty=False,
        K=2, assignment_strategy="round", label_loss="sigmoid")),
    "mm_greedy_k3_void": (1, 2, 11, 4, 8, 2, 5, 4, dict(
        smooth=1.0, sigmoid_scale=3.0, dice_scale=2.0, cls_scale=2.0, background_index=0,
        uncertainty_gamma=2.0, uncertainty_gamma_min=0.05, num_masks=3.0,
        force_unmatched_class_to_background=False, force_unmatched_masks_to_empty=False,
        K=3, assignment_strategy="greedy", void_class_index=4, label_loss="sigmoid")),
    "mm_pseudo_k2_softvoid": (1, 2, 10, 6, 6, 1, 6, 4, dict(
        smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
        uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, num_masks=None,
        force_unmatched_class_to_background=False, force_unmatched_masks_to_empty=False,
        K=2, assignment_strategy="pseudo_greedy", void_class_index=5, label_loss="softmax")),
    # s = 4 with rectangles off the 4-pixel grid: most boundary cells hold two
    # to four labels (mixed cells), a few more
    "mm_s4_mixed_uncert": (2, 2, 16, 6, 8, 4, 6, 8, dict(
        smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
        uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, num_masks=None,
        force_unmatched_class_to_background=True, force_unmatched_masks_to_empty=False,
        K=1, assignment_strategy="global", void_class_index=5, label_loss="softmax")),
}


def make_targets(g, B, Ht, Wt, G, C):
    """Label map: background 0, ids 1..G painted as rectangles in order (later
    ones occlude earlier ones); one id is left unpainted on purpose."""
    t = torch.zeros(B, Ht, Wt, dtype=torch.int64)
    for b in range(B):
        for gid in range(1, G + 1):
            if b == 1 and gid == G:  # absent GT -> +inf column in that image
                continue
            h = int(torch.randint(1, max(2, Ht // 2) + 1, (1,), generator=g))
            w = int(torch.randint(1, max(2, Wt // 2) + 1, (1,), generator=g))
            y0 = int(torch.randint(0, Ht - h + 1, (1,), generator=g))
            x0 = int(torch.randint(0, Wt - w + 1, (1,), generator=g))
            t[b, y0:y0 + h, x0:x0 + w] = gid
    y = torch.randint(0, C - 1, (B, G + 1), generator=g)
    y[:, 0] = -1
    return t, y


def params_for(kw, C):
    strategy = STRATS.index(kw.get("assignment_strategy", "global"))
    fg = float(kw.get("mask_focal_gamma", 0.0))
    fa = kw.get("mask_focal_alpha", None)
    fa = -1.0 if fa is None else float(fa)
    cg = kw.get("cls_focal_gamma", None)
    ca = kw.get("cls_focal_alpha", None)
    softmax = kw.get("label_loss", "sigmoid") == "softmax"
    return O.Params(
        smooth=kw["smooth"], sigmoid_scale=kw["sigmoid_scale"], dice_scale=kw["dice_scale"],
        cls_scale=kw["cls_scale"], background_index=kw["background_index"],
        uncertainty_gamma=kw["uncertainty_gamma"], uncertainty_gamma_min=kw["uncertainty_gamma_min"],
        num_masks=-1.0 if kw["num_masks"] is None else float(kw["num_masks"]),
        force_unmatched_class_to_background=kw["force_unmatched_class_to_background"],
        force_unmatched_masks_to_empty=kw["force_unmatched_masks_to_empty"],
        topk_matches=kw["K"], strategy_id=strategy, mask_gamma=fg, mask_alpha=fa,
        cls_gamma=fg if cg is None else float(cg), cls_alpha=fa if ca is None else float(ca),
        void_class_index=-1 if kw.get("void_class_index") is None else kw["void_class_index"],
        use_softmax_label_loss=softmax, normalize_uncertainty=True)


def gen_case(name, spec, seed):
    L, B, Q, H, W, s, C, G, kw = spec
    for attempt in range(50):
        g = torch.Generator().manual_seed(seed + 1000 * attempt)
        x32 = (torch.randn(L, B, Q, H, W, generator=g) * 3.0).float()
        z32 = torch.randn(L, B, Q, C, generator=g).float()
        t, y = make_targets(g, B, H * s, W * s, G, C)
        x = x32.double().requires_grad_(True)
        z = z32.double().requires_grad_(True)
        P = params_for(kw, C)
        py_kw = {k: v for k, v in kw.items()}
        out = RF.mask_matching_py(x, t, z, y, **py_kw)
        p2g, prd, m, d, c = out
        a = torch.rand(3, L, generator=g, dtype=torch.float64) + 0.5
        (a[0] * m + a[1] * d + a[2] * c).sum().backward()
        sep = RF.pairwise_mask_loss_py(
            x.detach(), t, z.detach(), y, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
            kw["cls_scale"], kw["background_index"], uncertainty_gamma=kw["uncertainty_gamma"],
            uncertainty_gamma_min=kw["uncertainty_gamma_min"],
            mask_focal_gamma=kw.get("mask_focal_gamma", 0.0),
            mask_focal_alpha=kw.get("mask_focal_alpha", None),
            cls_focal_gamma=kw.get("cls_focal_gamma", None) if kw.get("label_loss") != "softmax" else 0.0,
            cls_focal_alpha=kw.get("cls_focal_alpha", None) if kw.get("label_loss") != "softmax" else None,
            label_loss=kw.get("label_loss", "sigmoid"))
        # no-near-tie filter: the fp32-summed cost must give the same assignment
        # as the reference's float64 scipy solve, and a 1e-3 perturbation too.
        sep32 = sep.numpy().astype(np.float32)
        tot32 = (sep32[0] + sep32[1]) + sep32[2]
        ok = True
        rng = np.random.default_rng(seed + attempt)
        for l in range(L):
            for b in range(B):
                a1, _ = O.assign_slice(tot32[l, b].astype(np.float64), P.inf_thresh,
                                       P.topk_matches, P.strategy_id, use_ref=True)
                pert = tot32[l, b].astype(np.float64) * (1 + 1e-3 * rng.uniform(-1, 1, tot32[l, b].shape))
                a2, _ = O.assign_slice(pert, P.inf_thresh, P.topk_matches, P.strategy_id, use_ref=True)
                if not (np.array_equal(a1, p2g[l, b].numpy()) and np.array_equal(a1, a2)):
                    ok = False
        if ok:
            break
    else:
        raise RuntimeError(f"{name}: could not draw a tie-free case")
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        mask_logits=x32.numpy(), mask_targets=t.numpy(), cls_logits=z32.numpy(),
        cls_targets=y.numpy(), sep=sep.numpy(), pred_to_gt=p2g.numpy(), pred_round=prd.numpy(),
        layer_mask_mean=m.detach().numpy(), layer_dice_mean=d.detach().numpy(),
        layer_cls_mean=c.detach().numpy(), upstream=a.numpy(),
        grad_mask_logits=x.grad.numpy(), grad_cls_logits=z.grad.numpy(),
        params=np.array(repr(P.__dict__)), attempt=np.array(attempt))
    print(f"{name}: attempt {attempt}, matched {(p2g >= 0).sum().item()}")


def gen_solver(seed=7):
    rng = np.random.default_rng(seed)
    costs, meta, p2gs, prds = [], [], [], []
    shapes = [(12, 5), (20, 20), (7, 11), (30, 8), (16, 16), (40, 25)]
    for si, (Q, G) in enumerate(shapes):
        for variant in range(4):
            c = rng.random((Q, G))
            if variant == 1:
                c[:, rng.integers(0, G)] = np.inf  # all-inf column
                c[rng.random((Q, G)) < 0.2] = np.inf
            elif variant == 2:
                c = np.round(c * 4) / 4  # many exact ties
            elif variant == 3:
                c[rng.random((Q, G)) < 0.1] = np.nan
                c[rng.random((Q, G)) < 0.1] = 5e29
            for thr in (1e30, 0.6):
                for strat in range(4):
                    for K in range(4):
                        p2g, prd = O.assign_slice(c, thr, K, strat, use_ref=True)
                        costs.append(np.pad(c, ((0, 40 - Q), (0, 25 - G)), constant_values=-7.0))
                        meta.append((Q, G, strat, K, thr))
                        p2gs.append(np.pad(p2g, (0, 40 - Q), constant_values=-9))
                        prds.append(np.pad(prd, (0, 40 - Q), constant_values=-9))
    np.savez_compressed(os.path.join(HERE, "solver.npz"), costs=np.stack(costs),
                        meta=np.array(meta, dtype=np.float64), pred_to_gt=np.stack(p2gs),
                        pred_round=np.stack(prds))
    print("solver cases:", len(costs))


def gen_sampled(name, seed, L, B, Q, H, W, Ht, Wt, G, P, focal_gamma=0.0, focal_alpha=None,
                bg=0, align_corners=False):
    """Point-sampled costs of the reference's *_sampling_py functions
    (functions/sigmoid/pw_sigmoid_ce.py:407-549, functions/dice/pw_dice_loss.py:174-268);
    the coordinates are the ones those functions draw after torch.manual_seed(seed)."""
    from oracle import sampled as S
    g = torch.Generator().manual_seed(seed)
    x32 = (torch.randn(L, B, Q, H, W, generator=g) * 3.0).float()
    t, _ = make_targets(g, B, Ht, Wt, G, 3)
    x = x32  # the reference samples with fp32 coordinates, so it runs in fp32
    torch.manual_seed(seed)
    sce = RF.pairwise_sigmoid_cross_entropy_loss_sampling_py(
        x, t, background_index=bg, scale=2.0, num_points=P, align_corners=align_corners,
        focal_gamma=focal_gamma, focal_alpha=focal_alpha)
    torch.manual_seed(seed)
    dice = RF.pairwise_dice_loss_sampling_py(x, t, smooth=1.0, background_index=bg, scale=3.0,
                                             num_points=P, align_corners=align_corners)
    coords = S.reference_coords(t, P, seed, background_index=bg)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), mask_logits=x32.numpy(),
                        mask_targets=t.numpy(), coords=coords.numpy(), sce=sce.numpy(),
                        dice=dice.numpy(), meta=np.array([P, bg, int(align_corners), focal_gamma,
                                                          -1.0 if focal_alpha is None else focal_alpha]))
    print(f"{name}: sce finite {np.isfinite(sce.numpy()).sum()}")


if __name__ == "__main__":
    # python make_golden.py [case names ...]: all fixtures, or only the named
    # mm_* cases (each case keeps its seed, so a subset run writes the same files)
    O.build()
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref was not built: the reference sources are required")
    only = set(sys.argv[1:])
    for i, (name, spec) in enumerate(CASES.items()):
        if not only or name in only:
            gen_case(name, spec, 100 + i)
    if only:
        raise SystemExit(0)
    gen_solver()
    gen_sampled("sampled_basic", 501, 1, 3, 8, 12, 12, 24, 24, 5, 500)
    gen_sampled("sampled_focal_s4", 502, 2, 2, 6, 8, 10, 32, 40, 4, 777, focal_gamma=2.0,
                focal_alpha=0.25)
    gen_sampled("sampled_align_nobg", 503, 1, 2, 5, 9, 9, 9, 9, 3, 300, bg=-1, align_corners=True)
