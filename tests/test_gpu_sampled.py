"""GPU parity of the point-sampled path (config 3): costs against the
reference's *_sampling_py fixtures, bf16 logits and the matched losses and
gradients against the CPU restatement in oracle/sampled.py."""
import numpy as np
import pytest
import torch

from golden_cases import GOLDEN
from mask_loss_b200 import ops, synthetic
from mask_loss_b200 import functions as F
from oracle import oracle as O
from oracle import sampled as S

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def close(got, ref, rtol=1e-4, atol=1e-5):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    f = np.isfinite(ref)
    np.testing.assert_allclose(got[f], ref[f], rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", ["sampled_basic", "sampled_focal_s4", "sampled_align_nobg"])
def test_sampled_costs_golden(name):
    d = np.load(GOLDEN + f"/{name}.npz")
    Pn, bg, al, fg, fa = d["meta"]
    gt = int(d["mask_targets"].max()) + 1
    ml = torch.from_numpy(d["mask_logits"]).to(DEV)
    mt = torch.from_numpy(d["mask_targets"]).to(DEV)
    pc = torch.from_numpy(d["coords"]).to(DEV)
    L, B, Q = ml.shape[:3]
    cl = torch.zeros(L, B, Q, 1, device=DEV)
    ct = torch.full((B, gt), -1, dtype=torch.int64, device=DEV)
    out = ops.pairwise_mask_loss_sampled_forward(ml, mt, cl, ct, pc, 1.0, 2.0, 3.0, 1.0, int(bg),
                                                 float(fg), float(fa), 0.0, -1.0, False, bool(al))
    close(out[0].cpu().numpy(), d["sce"])
    close(out[1].cpu().numpy(), d["dice"])


def _case(seed, dtype, big=False):
    torch.manual_seed(seed)
    L, B, Q, H, W, s, C, Pn = 1, 3, 20, 16, 16, 4, 9, 777
    if big:  # 160x160 fp32 gradient map exceeds the shared-memory row path
        L, B, Q, H, W, s, C, Pn = 1, 2, 6, 160, 160, 1, 9, 1500
    cfg = synthetic.Config("pt", 12, L, B, Q, H, W, s, C, 3.0, "ellipse", ("fixed", 5), (0.02, 0.2))
    b = synthetic.make_batch(cfg)
    coords = torch.rand(B, Pn, 2)
    ml = b["mask_logits"]
    if dtype == torch.bfloat16:
        ml = ml.to(torch.bfloat16)
    return ml, b["mask_targets"], b["cls_logits"], b["cls_targets"], coords, C


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("variant", ["softmax", "sigmoid_focal_k2", "big_map"])
def test_sampled_matching_forward_backward(dtype, variant):
    ml, mt, cl, ct, pc, C = _case(7, dtype, big=variant == "big_map")
    kw = dict(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
              uncertainty_gamma=0.0, inf_thresh=1e30, num_masks=-1.0,
              force_unmatched_class_to_background=True, topk_matches=1, strategy_id=0,
              void_class_index=C - 1, use_softmax_label_loss=True)
    if variant == "sigmoid_focal_k2":
        kw.update(use_softmax_label_loss=False, mask_gamma=2.0, mask_alpha=0.25, cls_gamma=1.0,
                  cls_alpha=0.3, topk_matches=2, num_masks=4.0)
    P = O.Params(**kw)
    x = ml.to(DEV).requires_grad_(True)
    z = cl.to(DEV).requires_grad_(True)
    p2g, prd, m, d, c = F.MaskMatchingSampledFunction.apply(
        x, mt.to(DEV), z, ct.to(DEV), pc.to(DEV), P.smooth, P.sigmoid_scale, P.dice_scale,
        P.cls_scale, P.background_index, P.inf_thresh, None if P.num_masks <= 0 else P.num_masks,
        P.force_unmatched_class_to_background, P.topk_matches, "global", P.mask_gamma,
        None if P.mask_alpha < 0 else P.mask_alpha, P.cls_gamma,
        None if P.cls_alpha < 0 else P.cls_alpha, P.void_class_index,
        "softmax" if P.use_softmax_label_loss else "sigmoid")
    (1.0 * m + 0.7 * d + 1.3 * c).sum().backward()
    ep2g, eprd, emeans, esep, egm, egc = S.mask_matching_sampled(
        ml.float().numpy(), mt.numpy(), cl.numpy(), ct.numpy(), pc.numpy(), P,
        upstream=(1.0, 0.7, 1.3))
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    np.testing.assert_array_equal(prd.cpu().numpy(), eprd)
    close(torch.stack([m, d, c]).detach().cpu().numpy(), emeans)
    gm = x.grad.float().cpu().numpy()
    tol = 1e-5 if dtype == torch.float32 else 1e-2  # bf16 gradient storage
    np.testing.assert_allclose(gm, egm, rtol=max(1e-4, tol), atol=tol * np.abs(egm).max())
    np.testing.assert_allclose(z.grad.cpu().numpy(), egc, rtol=1e-4, atol=1e-5 * np.abs(egc).max())


def test_sampled_backward_without_forward_workspace():
    """The op-level backward rebuilds the sorted points itself when it is not
    handed the forward's workspace; both give the same gradients."""
    ml, mt, cl, ct, pc, C = _case(9, torch.float32)
    d = [t.to(DEV) for t in (ml, mt, cl, ct, pc)]
    args = (1.0, 5.0, 5.0, 2.0, 0, 1e30, -1.0, True, 1, 0, 0.0, -1.0, 0.0, -1.0, C - 1, True, False)
    p2g, prd, means, saved, _, fws = ops.mask_matching_sampled_ex(*d, *args, want_saved=True,
                                                                  want_workspace=True)
    g = torch.ones(1, device=DEV)
    bargs = (1.0, 5.0, 5.0, 2.0, 0, -1.0, True, 0.0, -1.0, 0.0, -1.0, C - 1, True, False)
    a = ops.mask_matching_sampled_backward(g, g, g, *d, p2g, saved, *bargs, forward_workspace=fws)
    b = ops.mask_matching_sampled_backward(g, g, g, *d, p2g, saved, *bargs)
    torch.testing.assert_close(a[0], b[0], rtol=1e-5, atol=1e-8)
    torch.testing.assert_close(a[1], b[1], rtol=0, atol=0)


def test_sampled_auto_num_masks_counts_present_gts():
    """num_masks="auto": the present non-background GT ids of the full label
    maps (not of the points), the same as passing that count."""
    ml, mt, cl, ct, pc, C = _case(11, torch.float32)
    d = [t.to(DEV) for t in (ml, mt, cl, ct, pc)]
    present = sum(int((torch.unique(mt[i]) > 0).sum()) for i in range(mt.shape[0]))

    def run(nm):
        x = d[0].clone().requires_grad_(True)
        z = d[2].clone().requires_grad_(True)
        p2g, prd, m, dd, c = F.MaskMatchingSampledFunction.apply(
            x, d[1], z, d[3], d[4], 1.0, 5.0, 5.0, 2.0, 0, 1e30, nm, False, 1, "global", 0.0,
            None, None, None, C - 1, "softmax")
        (m + dd + c).sum().backward()
        return torch.stack([m, dd, c]).detach(), x.grad, z.grad

    for u, v in zip(run("auto"), run(float(present))):
        torch.testing.assert_close(u, v, rtol=1e-6, atol=1e-9)
