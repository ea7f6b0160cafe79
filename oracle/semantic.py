"""CPU oracle of the standalone semantic losses.

TEST INFRASTRUCTURE ONLY (tests/); the product never imports it.

Restates in float64 numpy:
* sigmoid CE: sigmoid_cross_entropy_loss_py (functions/sigmoid/sigmoid_ce.py:147-226)
  and its gradient as src/cuda/sigmoid_ce.cu:116-205 writes it;
* dice: dice_loss_py (functions/dice/dice_loss.py:100-168), the I, P, T sums
  of src/cuda/dice_loss.cu:13-82 and the gradient of :84-157.
Labels outside [0, C) count for no class (the kernels' rule; the reference's
_py one-hot path cannot take them).  Pinned against fixtures made by the
reference functions (tests/golden/make_golden_semantic.py, ``semantic_*.npz``).
"""
from __future__ import annotations

import numpy as np


def _counts(targets, C, H, W):
    """(B, C, H, W) pixel counts of each class per low-res cell."""
    t = np.asarray(targets)
    B, Ht, Wt = t.shape
    s = Ht // H
    blocks = t.reshape(B, H, s, W, s).transpose(0, 1, 3, 2, 4).reshape(B, H, W, s * s)
    n = np.zeros((B, C, H, W))
    for c in range(C):
        n[:, c] = (blocks == c).sum(-1)
    return n, s


def _terms(x):
    x = np.asarray(x, np.float64)
    p = 1.0 / (1.0 + np.exp(-x))
    sp = np.log1p(np.exp(-np.abs(x)))
    return p, sp + np.maximum(-x, 0.0), sp + np.maximum(x, 0.0)  # p, ce_pos, ce_neg


def sigmoid_ce(logits, targets, num_masks, scale=1.0, gamma=0.0, alpha=-1.0, grad_out=None):
    """(loss (L,), grad (L,B,C,H,W) or None)."""
    x = np.asarray(logits, np.float64)
    L, B, C, H, W = x.shape
    n, s = _counts(targets, C, H, W)
    N2 = float(s * s)
    Ht, Wt = H * s, W * s
    ap = alpha if alpha >= 0 else 1.0
    an = 1.0 - alpha if alpha >= 0 else 1.0
    p, cp, cn = _terms(x)
    mp = (1.0 - p) ** gamma if gamma > 0 else np.ones_like(p)
    mn = p ** gamma if gamma > 0 else np.ones_like(p)
    loss_el = ap * mp * cp * n[None] + an * mn * cn * (N2 - n[None])
    loss = loss_el.sum(axis=(1, 2, 3, 4)) / (num_masks * Ht * Wt) * scale
    grad = None
    if grad_out is not None:
        g = (-ap * n[None] * mp * (gamma * p * cp + 1.0 - p) +
             an * (N2 - n[None]) * mn * (gamma * (1.0 - p) * cn + p))
        go = np.asarray(grad_out, np.float64) * scale / (num_masks * Ht * Wt)
        grad = g * go[:, None, None, None, None]
    return loss, grad


def dice(logits, targets, smooth, num_masks, scale=1.0, grad_out=None):
    """(loss (L,), I, P, T (L,B,C), grad or None)."""
    x = np.asarray(logits, np.float64)
    L, B, C, H, W = x.shape
    n, s = _counts(targets, C, H, W)
    N2 = float(s * s)
    p = 1.0 / (1.0 + np.exp(-x))
    I = (p * n[None]).sum(axis=(3, 4))
    P = N2 * p.sum(axis=(3, 4))
    T = np.broadcast_to(n.sum(axis=(2, 3))[None], I.shape).copy()
    d = (2.0 * I + smooth) / (P + T + smooth)
    loss = (1.0 - d).sum(axis=(1, 2)) / num_masks * scale
    grad = None
    if grad_out is not None:
        den = (P + T + smooth)[..., None, None]
        dd = (2.0 * n[None] * den - N2 * (2.0 * I + smooth)[..., None, None]) / den ** 2
        go = -np.asarray(grad_out, np.float64) / num_masks * scale
        grad = go[:, None, None, None, None] * dd * p * (1.0 - p)
    return loss, I, P, T, grad
