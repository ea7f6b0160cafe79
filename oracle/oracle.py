"""CPU oracle for the mask_loss matching + loss hot path.

TEST INFRASTRUCTURE ONLY.  This module is imported by ``tests/``, by
``__graft_entry__.smoke()`` (as the checker) and by ``bench.py``'s CPU arm.
The product package ``mask_loss_b200`` never imports it and has no CPU
fallback.

It wraps ``oracle/liboracle.so`` (the plain-C restatement in ``oracle.c``)
and, when it was built, ``oracle/_ref/libref.so`` (the reference's own C++
solver compiled from ``src/cpu/matching.cpp``).  All results are float64
numpy arrays.

``mask_matching`` mirrors the reference op ``mask_loss.mask_matching``
(``src/cpu/matching.cpp:592-752``): fused pairwise costs, fp32 cost sum,
per-slice assignment on the fp64 copy of that sum, matched-loss means.
``mask_matching_backward`` mirrors ``src/cuda/mask_matching_backward.cu:378-621``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None


def reference_root():
    """The reference checkout (AndyBarcia/mask_loss sources), or None.

    ``MASK_LOSS_REF`` names it; otherwise a ``reference`` directory beside the
    repository is used when it exists.  Only build steps and fixture
    generators look for it; tests, smoke() and bench.py never do."""
    root = os.environ.get("MASK_LOSS_REF")
    if not root:
        root = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")
    return root if os.path.isfile(os.path.join(root, "src", "cpu", "matching.cpp")) else None


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and oracle/_ref when the reference sources exist)."""
    cmd = ["make", "-C", _HERE]
    root = reference_root()
    if root:
        cmd.append("REF_SRC=" + os.path.join(root, "src"))
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout[-2000:] + out.stderr[-4000:])
    if not quiet:
        print(out.stdout[-500:])


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            subprocess.run(["make", "-C", _HERE, "liboracle.so"], check=True,
                           capture_output=True)
        _LIB = ctypes.CDLL(path)
    return _LIB


def ref_lib():
    """The reference C++ solver, or None when oracle/_ref was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libref.so")
        if not os.path.exists(path):
            return None
        try:
            _REF = ctypes.CDLL(path)
        except OSError:
            return None
    return _REF


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


I64 = ctypes.c_int64
F64 = ctypes.c_double


@dataclass
class Params:
    """The scalar arguments of ``mask_loss.mask_matching`` (src/bindings.cpp:86-111)."""
    smooth: float = 1.0
    sigmoid_scale: float = 1.0
    dice_scale: float = 1.0
    cls_scale: float = 1.0
    background_index: int = -1
    uncertainty_gamma: float = 1.0
    uncertainty_gamma_min: float = 0.05
    inf_thresh: float = 1e30
    num_masks: float = -1.0
    force_unmatched_class_to_background: bool = False
    force_unmatched_masks_to_empty: bool = False
    topk_matches: int = 1
    strategy_id: int = 0
    mask_gamma: float = 0.0
    mask_alpha: float = -1.0
    cls_gamma: float = 0.0
    cls_alpha: float = -1.0
    void_class_index: int = -1
    use_softmax_label_loss: bool = False
    normalize_uncertainty: bool = True


class _OrcParams(ctypes.Structure):
    _fields_ = [
        ("smooth", F64), ("sigmoid_scale", F64), ("dice_scale", F64), ("cls_scale", F64),
        ("background_index", I64), ("ug", F64), ("ugmin", F64), ("num_masks", F64),
        ("force_cls", ctypes.c_int), ("force_masks", ctypes.c_int),
        ("mask_gamma", F64), ("mask_alpha", F64), ("cls_gamma", F64), ("cls_alpha", F64),
        ("void_class_index", I64), ("use_softmax", ctypes.c_int),
        ("normalize_uncertainty", ctypes.c_int),
    ]


def _orc_params(P: Params) -> _OrcParams:
    return _OrcParams(P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale,
                      P.background_index, P.uncertainty_gamma, P.uncertainty_gamma_min,
                      P.num_masks, int(P.force_unmatched_class_to_background),
                      int(P.force_unmatched_masks_to_empty), P.mask_gamma, P.mask_alpha,
                      P.cls_gamma, P.cls_alpha, P.void_class_index,
                      int(P.use_softmax_label_loss), int(P.normalize_uncertainty))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def gt_out(GT_total: int, background_index: int) -> int:
    return GT_total - (1 if 0 <= background_index < GT_total else 0)


def label_counts(targets, H: int, W: int, GT_total: int):
    """(B,GT_total,H,W) int32 counts and (B,GT_total) totals (src/cuda/utils.cuh:6-36)."""
    t = _i64(targets)
    B, Ht, Wt = t.shape
    counts = np.zeros((B, GT_total, H, W), np.int32)
    totals = np.zeros((B, GT_total), np.int32)
    rc = lib().orc_label_counts(_p(t), I64(B), I64(Ht), I64(Wt), I64(H), I64(W),
                                I64(GT_total), _p(counts), _p(totals))
    if rc:
        raise ValueError("label_counts: bad shapes")
    return counts, totals


def pairwise_mask_cost(mask_logits, mask_targets, GT_total: int, P: Params) -> np.ndarray:
    """(2,L,B,Q,GT_out) BCE and dice costs (src/cuda/pw_mask.cu:52-449)."""
    x = _f32(mask_logits)
    t = _i64(mask_targets)
    L, B, Q, H, W = x.shape
    _, Ht, Wt = t.shape
    G = gt_out(GT_total, P.background_index)
    out = np.zeros((2, L, B, Q, G), np.float64)
    if G == 0:
        return out
    rc = lib().orc_pairwise_mask_cost(
        _p(x), _p(t), I64(L), I64(B), I64(Q), I64(H), I64(W), I64(Ht), I64(Wt),
        I64(GT_total), I64(P.background_index), F64(P.smooth), F64(P.sigmoid_scale),
        F64(P.dice_scale), F64(P.uncertainty_gamma), F64(P.uncertainty_gamma_min),
        F64(P.mask_gamma), F64(P.mask_alpha), ctypes.c_int(int(P.normalize_uncertainty)),
        _p(out))
    if rc:
        raise ValueError(f"pairwise_mask_cost failed ({rc})")
    return out


def pairwise_label_cost(cls_logits, cls_targets, P: Params, use_softmax=None,
                        scale=None, gamma=None, alpha=None) -> np.ndarray:
    """(L,B,Q,GT_out) label cost (src/cuda/pw_softmax_label_loss.cu:12-103,
    src/cuda/pw_sigmoid_label_loss.cu:16-106)."""
    z = _f32(cls_logits)
    y = _i64(cls_targets)
    L, B, Q, C = z.shape
    GT_total = y.shape[1]
    G = gt_out(GT_total, P.background_index)
    out = np.zeros((L, B, Q, G), np.float64)
    if G == 0:
        return out
    sm = P.use_softmax_label_loss if use_softmax is None else use_softmax
    rc = lib().orc_pairwise_label_cost(
        _p(z), _p(y), I64(L), I64(B), I64(Q), I64(C), I64(GT_total),
        I64(P.background_index), F64(P.cls_scale if scale is None else scale),
        F64(P.cls_gamma if gamma is None else gamma),
        F64(P.cls_alpha if alpha is None else alpha), ctypes.c_int(int(sm)), _p(out))
    if rc:
        raise ValueError("pairwise_label_cost failed")
    return out


def pairwise_mask_loss(mask_logits, mask_targets, cls_logits, cls_targets, P: Params):
    """(3,L,B,Q,GT_out): the output of ``pairwise_mask_loss_forward``."""
    GT_total = np.asarray(cls_targets).shape[1]
    mc = pairwise_mask_cost(mask_logits, mask_targets, GT_total, P)
    lc = pairwise_label_cost(cls_logits, cls_targets, P)
    return np.concatenate([mc, lc[None]], axis=0)


def assign_slice(cost, inf_thresh: float, topk: int, strategy: int, use_ref: bool = False):
    """pred_to_gt, pred_round (int64, (Q,)) for one fp64 (Q,GT_out) slice.

    use_ref=True runs the reference's compiled solver (oracle/_ref)."""
    c = np.ascontiguousarray(np.asarray(cost, dtype=np.float64))
    Q, G = c.shape
    p2g = np.empty(Q, np.int64)
    prd = np.empty(Q, np.int64)
    L = ref_lib() if use_ref else lib()
    if L is None:
        raise RuntimeError("oracle/_ref was not built")
    fn = L.ref_assign_slice if use_ref else L.orc_assign_slice
    rc = fn(_p(c), I64(Q), I64(G), F64(inf_thresh), I64(topk), ctypes.c_int(strategy),
            _p(p2g), _p(prd))
    if rc:
        raise RuntimeError("Hungarian: no augmenting path found; check costs/inf_thresh.")
    return p2g, prd


def assign_batch_ref(costs, inf_thresh, topk, strategy, threads):
    """Reference solver over all (N,Q,G) slices on `threads` host threads."""
    c = np.ascontiguousarray(np.asarray(costs, dtype=np.float64))
    N, Q, G = c.shape
    p2g = np.empty((N, Q), np.int64)
    prd = np.empty((N, Q), np.int64)
    rc = ref_lib().ref_assign_batch(_p(c), I64(N), I64(Q), I64(G), F64(inf_thresh),
                                    I64(topk), ctypes.c_int(strategy), _p(p2g), _p(prd),
                                    ctypes.c_int(threads))
    if rc:
        raise RuntimeError("reference solver failed")
    return p2g, prd


def match(costs_f32, P: Params, use_ref: bool = False):
    """Assign every (l,b) slice of an fp32 (L,B,Q,GT_out) total cost."""
    c = np.asarray(costs_f32, dtype=np.float32).astype(np.float64)
    L, B, Q, G = c.shape
    p2g = np.full((L, B, Q), -1, np.int64)
    prd = np.full((L, B, Q), -1, np.int64)
    for l in range(L):
        for b in range(B):
            p2g[l, b], prd[l, b] = assign_slice(c[l, b], P.inf_thresh, P.topk_matches,
                                                P.strategy_id, use_ref=use_ref)
    return p2g, prd


def matched_loss_fwd(mask_logits, mask_targets, cls_logits, sep, p2g, P: Params):
    x = _f32(mask_logits)
    z = _f32(cls_logits)
    s = np.ascontiguousarray(np.asarray(sep, np.float64))
    pg = _i64(p2g)
    L, B, Q, H, W = x.shape
    _, Ht, Wt = np.asarray(mask_targets).shape
    C = z.shape[3]
    G = s.shape[4]
    out = np.zeros((3, L), np.float64)
    op = _orc_params(P)
    lib().orc_matched_loss_fwd(_p(x), _p(z), _p(s), _p(pg), I64(L), I64(B), I64(Q), I64(H),
                               I64(W), I64(Ht), I64(Wt), I64(C), I64(G), ctypes.byref(op),
                               _p(out))
    return out[0], out[1], out[2]


def mask_matching(mask_logits, mask_targets, cls_logits, cls_targets, P: Params,
                  use_ref: bool = False):
    """Oracle of ``mask_loss.mask_matching``.  Returns pred_to_gt, pred_round,
    layer_mask_mean, layer_dice_mean, layer_cls_mean and the (3,...) costs."""
    sep = pairwise_mask_loss(mask_logits, mask_targets, cls_logits, cls_targets, P)
    sep32 = sep.astype(np.float32)
    total = (sep32[0] + sep32[1]) + sep32[2]  # fp32 sum, src/cpu/matching.cpp:665
    p2g, prd = match(total, P, use_ref=use_ref)
    m, d, c = matched_loss_fwd(mask_logits, mask_targets, cls_logits, sep, p2g, P)
    return p2g, prd, m, d, c, sep


def mask_matching_backward(gm, gd, gc, mask_logits, mask_targets, cls_logits, cls_targets,
                           p2g, P: Params):
    x = _f32(mask_logits)
    t = _i64(mask_targets)
    z = _f32(cls_logits)
    y = _i64(cls_targets)
    pg = _i64(p2g)
    L, B, Q, H, W = x.shape
    _, Ht, Wt = t.shape
    C = z.shape[3]
    GT_total = y.shape[1]
    g = [np.ascontiguousarray(np.asarray(v, np.float64).reshape(L)) for v in (gm, gd, gc)]
    gx = np.zeros(x.shape, np.float64)
    gz = np.zeros(z.shape, np.float64)
    op = _orc_params(P)
    rc = lib().orc_matched_loss_bwd(_p(g[0]), _p(g[1]), _p(g[2]), _p(x), _p(t), _p(z), _p(y),
                                    _p(pg), I64(L), I64(B), I64(Q), I64(H), I64(W), I64(Ht),
                                    I64(Wt), I64(C), I64(GT_total), ctypes.byref(op), _p(gx),
                                    _p(gz))
    if rc:
        raise ValueError("matched_loss_bwd: bad shapes")
    return gx, gz
