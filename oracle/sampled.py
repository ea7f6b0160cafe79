"""CPU oracle of the point-sampled matching costs and losses (config 3).

TEST INFRASTRUCTURE ONLY (tests/, bench.py's CPU arm); the product never
imports it.

* ``reference_coords`` replays the random points the reference draws:
  ``torch.rand(1, P, 2)`` once per image that holds a non-background GT id, in
  image order (functions/sigmoid/pw_sigmoid_ce.py:488-504,
  functions/dice/pw_dice_loss.py:221-236).
* ``pairwise_costs_sampled`` restates pairwise_sigmoid_cross_entropy_loss_sampling_py
  (functions/sigmoid/pw_sigmoid_ce.py:407-549) and pairwise_dice_loss_sampling_py
  (functions/dice/pw_dice_loss.py:174-268) in float64 torch on the CPU:
  bilinear ``grid_sample`` of the logits (zero padding), floor-nearest label
  lookup ``ix = floor(x * (W_t - 1))`` in fp32, BCE = (<c+, t> + <c-, 1-t>)/P,
  dice = 1 - (2<p,t> + smooth)/(sum p + sum t + smooth), +inf for GT ids absent
  from the whole label map.  Pinned against fixtures made by the reference
  functions (tests/golden/make_golden.py, ``sampled_*.npz``).
* ``mask_matching_sampled`` chains those costs, the label cost and the fp32
  total into the C solver (oracle.c, pinned to the reference solver) and
  computes the matched losses and dL/dlogits with torch autograd.  The
  reference never wires point sampling into matching
  (functions/mask/matching.py:836), so this matched part is a restatement:
  parity unpinned beyond its pinned cost formula.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import oracle as O


def reference_coords(targets: torch.Tensor, num_points: int, seed: int, background_index=0):
    """(B, P, 2) float32 coordinates in [0,1) as the reference draws them on
    the CPU generator after torch.manual_seed(seed); rows of images without a
    non-background GT id are zero (the reference draws none for them)."""
    torch.manual_seed(seed)
    B = targets.shape[0]
    out = torch.zeros(B, num_points, 2, dtype=torch.float32)
    for b in range(B):
        ids = torch.unique(targets[b]).tolist()
        ids = [k for k in ids if k != background_index]
        if not ids:
            continue
        out[b] = torch.rand(1, num_points, 2)[0]
    return out


def _sample(logits, coords, align_corners):
    """(L,B,Q,P) bilinear samples of (L,B,Q,H,W) logits at (B,P,2) points."""
    L, B, Q, H, W = logits.shape
    P = coords.shape[1]
    out = torch.empty(L, B, Q, P, dtype=logits.dtype)
    for b in range(B):
        z = logits[:, b].reshape(L * Q, 1, H, W)
        grid = (2.0 * coords[b].to(logits.dtype) - 1.0).reshape(1, P, 1, 2).expand(L * Q, P, 1, 2)
        s = F.grid_sample(z, grid, align_corners=align_corners).reshape(L, Q, P)
        out[:, b] = s
    return out


def _point_labels(targets, coords):
    B, Ht, Wt = targets.shape
    x = coords[..., 0].float()
    y = coords[..., 1].float()
    ix = torch.clamp((x * (Wt - 1)).long(), 0, Wt - 1)
    iy = torch.clamp((y * (Ht - 1)).long(), 0, Ht - 1)
    return torch.stack([targets[b][iy[b], ix[b]] for b in range(B)])  # (B, P)


def pairwise_costs_sampled(mask_logits, mask_targets, coords, GT_total, P: O.Params,
                           align_corners=False, logits_grad=False):
    """(2,L,B,Q,GT_out) float64 BCE and dice point costs (torch tensors)."""
    z = torch.as_tensor(mask_logits).double()
    if logits_grad:
        z.requires_grad_(True)
    t = torch.as_tensor(mask_targets).long()
    c = torch.as_tensor(coords).float()
    L, B, Q = z.shape[:3]
    Np = c.shape[1]
    bg = P.background_index
    gcols = [k for k in range(GT_total) if not (0 <= bg < GT_total and k == bg)]
    G = len(gcols)
    zs = _sample(z, c, align_corners)  # (L,B,Q,Np)
    lab = _point_labels(t, c)  # (B,Np)
    ap = P.mask_alpha if P.mask_alpha >= 0 else 1.0
    an = 1.0 - P.mask_alpha if P.mask_alpha >= 0 else 1.0
    prob = torch.sigmoid(zs)
    mp = (1 - prob) ** P.mask_gamma if P.mask_gamma > 0 else torch.ones_like(prob)
    mn = prob ** P.mask_gamma if P.mask_gamma > 0 else torch.ones_like(prob)
    pos = ap * mp * F.softplus(-zs)
    neg = an * mn * F.softplus(zs)
    onehot = torch.stack([(lab == k).double() for k in gcols], -1)  # (B,Np,G)
    tp = torch.einsum("lbqp,bpg->lbqg", pos, onehot)
    tn = torch.einsum("lbqp,bpg->lbqg", neg, 1.0 - onehot)
    bce = (tp + tn) / Np * P.sigmoid_scale
    inter = torch.einsum("lbqp,bpg->lbqg", prob, onehot)
    psum = prob.sum(-1, keepdim=True)
    tsum = onehot.sum(1)[None, :, None, :]
    dice = (1.0 - (2.0 * inter + P.smooth) / (psum + tsum + P.smooth)) * P.dice_scale
    present = torch.stack([torch.tensor([(t[b] == k).any().item() for k in gcols])
                           for b in range(B)])[None, :, None, :].expand(L, B, Q, G)
    inf = torch.full_like(bce, float("inf"))
    bce = torch.where(present, bce, inf)
    dice = torch.where(present, dice, inf)
    out = torch.stack([bce, dice])
    return (out, z) if logits_grad else out


def mask_matching_sampled(mask_logits, mask_targets, cls_logits, cls_targets, coords,
                          P: O.Params, align_corners=False, upstream=(1.0, 1.0, 1.0)):
    """Oracle of the sampled matching op: returns pred_to_gt, pred_round,
    (3,L) layer means, (3,L,B,Q,G) costs, grad_mask_logits, grad_cls_logits
    (grads of sum_l a*mask + b*dice + c*cls with `upstream` = (a, b, c))."""
    GT_total = np.asarray(cls_targets).shape[1]
    (mc, zt) = pairwise_costs_sampled(mask_logits, mask_targets, coords, GT_total, P,
                                      align_corners, logits_grad=True)
    lc = torch.as_tensor(O.pairwise_label_cost(cls_logits, cls_targets, P))
    sep = torch.cat([mc, lc[None]], 0)
    sep32 = sep.detach().float()
    total = (sep32[0] + sep32[1]) + sep32[2]
    p2g, prd = O.match(total.numpy(), P)
    L, B, Q = sep.shape[1:4]
    zc = torch.as_tensor(cls_logits).double().requires_grad_(True)
    # matched losses (gather) + unmatched class terms; denominators as in
    # src/cuda/mask_matching_forward.cu:549-578
    m = torch.as_tensor(p2g) >= 0
    idx = torch.as_tensor(p2g).clamp(min=0)[..., None]
    sep_g = torch.cat([mc, torch.as_tensor(
        O.pairwise_label_cost(cls_logits, cls_targets, P))[None]], 0)
    # class cost must be differentiable in the class logits: recompute it
    cl = _label_cost_torch(zc, torch.as_tensor(cls_targets), P)
    costs = torch.stack([mc[0], mc[1], cl])
    gathered = torch.gather(costs, 4, idx[None].expand(3, L, B, Q, 1))[..., 0]
    gathered = torch.where(m[None], gathered, torch.zeros_like(gathered))
    sums = gathered.sum((2, 3))  # (3, L)
    C = zc.shape[-1]
    has_void = 0 <= P.void_class_index < C
    if P.force_unmatched_class_to_background or has_void:
        um = _unmatched_cls_torch(zc, P) * P.cls_scale
        sums = sums + torch.stack([torch.zeros(L, dtype=torch.float64), torch.zeros(L, dtype=torch.float64),
                                   torch.where(~m, um, torch.zeros_like(um)).sum((1, 2))])
    matched = m.sum((1, 2)).double()
    tot = float(B * Q)
    nm = float(np.float32(P.num_masks)) if P.num_masks > 0 else None
    md = torch.full((L,), tot) if P.force_unmatched_masks_to_empty else (
        torch.full((L,), nm) if nm else matched)
    cd = torch.full((L,), tot) if (P.force_unmatched_class_to_background or has_void) else (
        torch.full((L,), nm) if nm else matched)
    means = torch.stack([sums[0] / md.clamp(min=1), sums[1] / md.clamp(min=1),
                         sums[2] / cd.clamp(min=1)])
    a = torch.tensor(upstream, dtype=torch.float64)[:, None]
    (a * means).sum().backward()
    return p2g, prd, means.detach().numpy(), sep.detach().numpy(), zt.grad.numpy(), zc.grad.numpy()


def _label_cost_torch(z, y, P):
    L, B, Q, C = z.shape
    bg = P.background_index
    GT = y.shape[1]
    keep = [k for k in range(GT) if not (0 <= bg < GT and k == bg)]
    T = y[:, keep]
    valid = (T >= 0) & (T < C)
    Tc = T.clamp(0, C - 1)
    if P.use_softmax_label_loss:
        lp = torch.log_softmax(z, -1)
        out = -torch.gather(lp, 3, Tc[None, :, None, :].expand(L, B, Q, T.shape[1]))
    else:
        ap = P.cls_alpha if P.cls_alpha >= 0 else 1.0
        an = 1.0 - P.cls_alpha if P.cls_alpha >= 0 else 1.0
        pr = torch.sigmoid(z)
        mp = (1 - pr) ** P.cls_gamma if P.cls_gamma > 0 else torch.ones_like(pr)
        mn = pr ** P.cls_gamma if P.cls_gamma > 0 else torch.ones_like(pr)
        pos = ap * mp * F.softplus(-z)
        neg = an * mn * F.softplus(z)
        idx = Tc[None, :, None, :].expand(L, B, Q, T.shape[1])
        out = (neg.sum(-1, keepdim=True) + torch.gather(pos, 3, idx) - torch.gather(neg, 3, idx)) / C
    out = out * P.cls_scale
    return torch.where(valid[None, :, None, :], out, torch.full_like(out, float("inf")))


def _unmatched_cls_torch(z, P):
    C = z.shape[-1]
    vi = P.void_class_index
    has_void = 0 <= vi < C
    if P.use_softmax_label_loss and P.force_unmatched_class_to_background and has_void:
        return -torch.log_softmax(z, -1)[..., vi]
    g = 0.0 if P.use_softmax_label_loss else P.cls_gamma
    al = -1.0 if P.use_softmax_label_loss else P.cls_alpha
    ap = al if al >= 0 else 1.0
    an = 1.0 - al if al >= 0 else 1.0
    pr = torch.sigmoid(z)
    mp = (1 - pr) ** g if g > 0 else torch.ones_like(pr)
    mn = pr ** g if g > 0 else torch.ones_like(pr)
    pos = ap * mp * F.softplus(-z)
    neg = an * mn * F.softplus(z)
    if P.force_unmatched_class_to_background:
        out = neg.mean(-1)
        if has_void:
            out = out + (pos[..., vi] - neg[..., vi]) / C
        return out
    return pos[..., vi]
