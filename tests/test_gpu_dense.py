"""Dense per-GT mask targets (B, GT_total, H_t, W_t), overlap allowed.  On
non-overlapping masks the results equal the label-map path; with overlaps
they match the dense oracle (oracle/dense.py).  Tolerances as elsewhere:
costs and losses 1e-4 relative / 1e-5 absolute, gradients 1e-5 of the
tensor's largest magnitude, identical +inf pattern, equal indices."""
import numpy as np
import pytest
import torch

from mask_loss_b200 import functions as F
from mask_loss_b200 import ops, synthetic
from oracle import dense as D
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def close(got, ref, rtol=1e-4, atol=1e-5):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert np.array_equal(np.isinf(got), np.isinf(ref)), "inf pattern differs"
    f = np.isfinite(ref)
    np.testing.assert_allclose(got[f], ref[f], rtol=rtol, atol=atol)


def close_grad(got, ref):
    ref = np.asarray(ref, np.float64)
    np.testing.assert_allclose(np.asarray(got, np.float64), ref, rtol=1e-4,
                               atol=1e-5 * max(np.abs(ref).max(), 1e-30))


def _fn_args(P):
    return (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
            P.uncertainty_gamma, P.uncertainty_gamma_min, P.normalize_uncertainty, P.inf_thresh,
            None if P.num_masks <= 0 else P.num_masks, P.force_unmatched_class_to_background,
            P.force_unmatched_masks_to_empty, P.topk_matches,
            ["global", "round", "greedy", "pseudo_greedy"][P.strategy_id], P.mask_gamma,
            None if P.mask_alpha < 0 else P.mask_alpha, P.cls_gamma,
            None if P.cls_alpha < 0 else P.cls_alpha,
            None if P.void_class_index < 0 else P.void_class_index,
            "softmax" if P.use_softmax_label_loss else "sigmoid")


def _run(ml, mt, cl, ct, P, up=(1.0, 0.7, 1.3)):
    x = ml.clone().requires_grad_(True)
    z = cl.clone().requires_grad_(True)
    p2g, prd, m, d, c = F.MaskMatchingFunction.apply(x, mt, z, ct, *_fn_args(P))
    (up[0] * m + up[1] * d + up[2] * c).sum().backward()
    return p2g, prd, torch.stack([m, d, c]).detach(), x.grad, z.grad


def test_dense_equals_label_map_without_overlap():
    cfg = synthetic.CONFIGS["cfg1"]
    b = synthetic.make_batch(cfg, device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    GT = ct.shape[1]
    masks = torch.stack([mt == g for g in range(GT)], 1).to(torch.uint8).contiguous()
    for ug in (0.0, 1.0):
        P = O.Params(**synthetic.parity_kwargs(cfg, uncertainty_gamma=ug))
        kw = list(synthetic.parity_kwargs(cfg, uncertainty_gamma=ug).values())
        a = ops.pairwise_mask_loss_forward(ml, mt, cl, ct, *[kw[i] for i in (0, 1, 2, 3, 4, 5, 6)],
                                           use_softmax_label_loss=True)
        d = ops.pairwise_mask_loss_forward(ml, masks, cl, ct, *[kw[i] for i in (0, 1, 2, 3, 4, 5, 6)],
                                           use_softmax_label_loss=True)
        close(d.cpu().numpy(), a.cpu().numpy())
        ra = _run(ml, mt, cl, ct, P)
        rd = _run(ml, masks, cl, ct, P)
        assert torch.equal(ra[0], rd[0]) and torch.equal(ra[1], rd[1])
        close(rd[2].cpu().numpy(), ra[2].cpu().numpy())
        close_grad(rd[3].cpu().numpy(), ra[3].cpu().numpy())
        close_grad(rd[4].cpu().numpy(), ra[4].cpu().numpy())


def _overlap_case(seed, L, B, Q, H, W, s, C, GT):
    rng = np.random.default_rng(seed)
    Ht, Wt = H * s, W * s
    yy, xx = np.mgrid[0:Ht, 0:Wt]
    masks = np.zeros((B, GT, Ht, Wt), np.uint8)
    for b in range(B):
        for g in range(1, GT - 1):  # column 0 background, last column left empty (absent)
            cy, cx = rng.uniform(0, Ht), rng.uniform(0, Wt)
            ry, rx = rng.uniform(1, Ht / 2), rng.uniform(1, Wt / 2)
            masks[b, g] = (((yy - cy) / ry) ** 2 + ((xx - cx) / rx) ** 2 <= 1.0)
    ml = (rng.standard_normal((L, B, Q, H, W)) * 3).astype(np.float32)
    cl = rng.standard_normal((L, B, Q, C)).astype(np.float32)
    ct = np.full((B, GT), -1, np.int64)
    ct[:, 1:] = rng.integers(0, C - 1, (B, GT - 1))
    return ml, masks, cl, ct


@pytest.mark.parametrize("variant", ["softmax", "unc_sigmoid_focal", "s2_forced_k2", "s3_unc_nobg",
                                     "masks_b_two_layers", "masks_b_two_query_tiles"])
def test_dense_overlapping_against_oracle(variant):
    if variant == "softmax":
        shp = (2, 2, 12, 8, 9, 1, 7, 6)
        P = O.Params(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                     background_index=0, uncertainty_gamma=0.0, force_unmatched_class_to_background=True,
                     void_class_index=6, use_softmax_label_loss=True)
    elif variant == "unc_sigmoid_focal":
        shp = (1, 3, 10, 6, 10, 1, 5, 5)
        P = O.Params(smooth=1.0, sigmoid_scale=2.0, dice_scale=3.0, cls_scale=1.5,
                     background_index=0, uncertainty_gamma=1.0, num_masks=4.0, mask_gamma=2.0,
                     mask_alpha=0.25, cls_gamma=1.5, cls_alpha=0.3)
    elif variant.startswith("masks_b"):
        # fp32 logits, s = 1, 16-cell rows, few GTs: the tf32 kernel with the
        # masks as its B operand, which also sums the mask areas -- once per
        # image over two layers, and over two query tiles
        shp = (2, 2, 12, 8, 8, 1, 7, 6) if variant.endswith("layers") else (1, 1, 130, 8, 8, 1, 7, 6)
        P = O.Params(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                     background_index=0, uncertainty_gamma=0.0, force_unmatched_class_to_background=True,
                     void_class_index=6, use_softmax_label_loss=True)
    elif variant == "s3_unc_nobg":
        shp = (2, 2, 9, 5, 7, 3, 4, 6)
        P = O.Params(smooth=0.5, sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0,
                     background_index=-1, uncertainty_gamma=1.0, uncertainty_gamma_min=0.1,
                     strategy_id=1, topk_matches=2)
    else:
        shp = (1, 2, 14, 6, 6, 2, 6, 5)
        P = O.Params(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                     background_index=0, uncertainty_gamma=0.0, force_unmatched_class_to_background=True,
                     force_unmatched_masks_to_empty=True, topk_matches=2, void_class_index=5,
                     use_softmax_label_loss=True)
    ml, masks, cl, ct = _overlap_case(sum(shp), *shp)
    assert (masks.sum(1) > 1).any(), "the case must contain overlaps"
    ep2g, eprd, em, ed, ec, esep = D.mask_matching(ml, masks, cl, ct, P)
    L = ml.shape[0]
    up = (1.0, 0.7, 1.3)
    egx, egz = D.mask_matching_backward(np.full(L, up[0]), np.full(L, up[1]), np.full(L, up[2]),
                                        ml, masks, cl, ct, ep2g, P)
    t = [torch.from_numpy(v).to(DEV) for v in (ml, masks, cl, ct)]
    kw = (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
          P.uncertainty_gamma, P.uncertainty_gamma_min)
    sep = ops.pairwise_mask_loss_forward(*t, *kw, mask_gamma=P.mask_gamma, mask_alpha=P.mask_alpha,
                                         cls_gamma=P.cls_gamma, cls_alpha=P.cls_alpha,
                                         use_softmax_label_loss=P.use_softmax_label_loss)
    close(sep.cpu().numpy(), esep)
    p2g, prd, means, gx, gz = _run(*t, P, up)
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    np.testing.assert_array_equal(prd.cpu().numpy(), eprd)
    close(means.cpu().numpy(), np.stack([em, ed, ec]))
    close_grad(gx.cpu().numpy(), egx)
    close_grad(gz.cpu().numpy(), egz)


def test_dense_backward_needs_saved_statistics():
    ml, masks, cl, ct = _overlap_case(3, 1, 1, 4, 4, 4, 1, 3, 3)
    t = [torch.from_numpy(v).to(DEV) for v in (ml, masks, cl, ct)]
    p2g = torch.zeros((1, 1, 4), dtype=torch.int64, device=DEV)
    g = torch.ones(1, device=DEV)
    with pytest.raises(RuntimeError, match="saved"):
        ops.mask_matching_backward(g, g, g, *t, p2g, 1.0, 1.0, 1.0, 1.0, 0, 0.0, 0.05, -1.0, False,
                                   False, 0.0, -1.0, 0.0, -1.0, -1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shp", [(2, 2, 12, 8, 12, 1, 7, 6), (1, 2, 10, 5, 7, 2, 6, 5)])
def test_dense_half_logits_equal_fp32_path_on_widened_values(dtype, shp):
    # 16-bit logits with overlapping masks: the dense kernel widens each value
    # (8-byte loads when H*W % 4 == 0, scalar loads otherwise) and runs the
    # fp32 arithmetic, so everything equals the fp32 run on the widened tensor
    ml, masks, cl, ct = _overlap_case(7 + sum(shp), *shp)
    P = O.Params(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                 background_index=0, uncertainty_gamma=1.0,
                 force_unmatched_class_to_background=True, void_class_index=shp[6] - 1,
                 use_softmax_label_loss=True)
    x16 = torch.from_numpy(ml).to(DEV).to(dtype)
    t = [torch.from_numpy(v).to(DEV) for v in (masks, cl, ct)]
    r16 = _run(x16, *t, P)
    r32 = _run(x16.float(), *t, P)
    assert torch.equal(r16[0], r32[0]) and torch.equal(r16[1], r32[1])
    assert torch.equal(r16[2], r32[2])
    assert r16[3].dtype == dtype
    assert torch.equal(r16[3], r32[3].to(dtype))
    assert torch.equal(r16[4], r32[4])


@pytest.mark.parametrize("gt", [6, 40])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_dense_tensor_core_path_with_half_logits_against_oracle(dtype, gt):
    # no entropy weights or focal terms: the tensor-core kernel runs (bf16
    # logits: the MMA reads the logits tile itself as its A operand; fp16:
    # bf16 hi/lo split).  Against the oracle on the widened logits: costs,
    # means and the class gradient at the usual tolerance, indices equal, the
    # mask gradient (stored in the logits' 16-bit type) within its rounding.
    # gt 6: the mask bytes are the B operand (bf16; tf32 for fp32 logits);
    # gt 40 (N = 48): counts as B, and fp32 logits on the bf16 hi/lo kernel
    shp = (2, 2, 12, 8, 8, 1, 7, gt)
    ml, masks, cl, ct = _overlap_case(41, *shp)
    P = O.Params(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                 background_index=0, uncertainty_gamma=0.0, force_unmatched_class_to_background=True,
                 void_class_index=shp[6] - 1, use_softmax_label_loss=True)
    x16 = torch.from_numpy(ml).to(DEV).to(dtype)
    wide = x16.float().cpu().numpy()
    ep2g, eprd, em, ed, ec, esep = D.mask_matching(wide, masks, cl, ct, P)
    L = ml.shape[0]
    up = (1.0, 0.7, 1.3)
    egx, egz = D.mask_matching_backward(np.full(L, up[0]), np.full(L, up[1]), np.full(L, up[2]),
                                        wide, masks, cl, ct, ep2g, P)
    t = [torch.from_numpy(v).to(DEV) for v in (masks, cl, ct)]
    kw = (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
          P.uncertainty_gamma, P.uncertainty_gamma_min)
    sep = ops.pairwise_mask_loss_forward(x16, *t, *kw, use_softmax_label_loss=True)
    close(sep.cpu().numpy(), esep)
    p2g, prd, means, gx, gz = _run(x16, *t, P, up)
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    close(means.cpu().numpy(), np.stack([em, ed, ec]))
    assert gx.dtype == dtype
    ref = np.asarray(egx, np.float64)
    if dtype == torch.float32:
        close_grad(gx.cpu().numpy(), ref)
    else:
        np.testing.assert_allclose(gx.float().cpu().numpy(), ref, rtol=1e-2,
                                   atol=1e-2 * np.abs(ref).max())
    close_grad(gz.cpu().numpy(), egz)
