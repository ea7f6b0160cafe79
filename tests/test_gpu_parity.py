"""GPU parity of the CUDA path against the CPU oracle and the reference's
golden fixtures.  Tolerances follow the stated contract: costs, losses and
gradients within 1e-4 relative / 1e-5 absolute (gradients: absolute bound
1e-5 of the tensor's largest magnitude), identical +inf pattern, bit-exact
assignment indices."""
import numpy as np
import pytest
import torch

from golden_cases import GOLDEN, case_names, load
from mask_loss_b200 import ops, synthetic
from mask_loss_b200 import functions as F
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5
DEV = "cuda:0"


def close(got, ref, rtol=RTOL, atol=ATOL, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.array_equal(np.isinf(got), np.isinf(ref)), f"{what}: inf pattern differs"
    f = np.isfinite(ref)
    np.testing.assert_allclose(got[f], ref[f], rtol=rtol, atol=atol, err_msg=what)


def close_grad(got, ref, what=""):
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    np.testing.assert_allclose(np.asarray(got, np.float64), ref, rtol=RTOL, atol=1e-5 * scale,
                               err_msg=what)


def to_dev(d):
    return (torch.from_numpy(d["mask_logits"]).to(DEV), torch.from_numpy(d["mask_targets"]).to(DEV),
            torch.from_numpy(d["cls_logits"]).to(DEV), torch.from_numpy(d["cls_targets"]).to(DEV))


def op_args(P: O.Params):
    return (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
            P.uncertainty_gamma, P.uncertainty_gamma_min, P.inf_thresh, P.num_masks,
            P.force_unmatched_class_to_background, P.force_unmatched_masks_to_empty,
            P.topk_matches, P.strategy_id, P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha,
            P.void_class_index, P.use_softmax_label_loss, P.normalize_uncertainty)


def bwd_args(P: O.Params):
    return (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
            P.uncertainty_gamma, P.uncertainty_gamma_min, P.num_masks,
            P.force_unmatched_class_to_background, P.force_unmatched_masks_to_empty,
            P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha, P.void_class_index,
            P.use_softmax_label_loss, P.normalize_uncertainty)


# --------------------------------------------------------------------------
# golden fixtures (reference Python path, float64)
# --------------------------------------------------------------------------
@pytest.mark.parametrize("name", case_names())
def test_golden_costs(name):
    d, P = load(name)
    ml, mt, cl, ct = to_dev(d)
    out = ops.pairwise_mask_loss_forward(
        ml, mt, cl, ct, P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
        P.uncertainty_gamma, P.uncertainty_gamma_min, P.mask_gamma, P.mask_alpha, P.cls_gamma,
        P.cls_alpha, P.use_softmax_label_loss, P.normalize_uncertainty)
    close(out.cpu().numpy(), d["sep"], what=name)


@pytest.mark.parametrize("name", case_names())
def test_golden_matching_forward_backward(name):
    d, P = load(name)
    ml, mt, cl, ct = to_dev(d)
    ml.requires_grad_(True)
    cl.requires_grad_(True)
    strat = ["global", "round", "greedy", "pseudo_greedy"][P.strategy_id]
    p2g, prd, m, dd, c = F.MaskMatchingFunction.apply(
        ml, mt, cl, ct, P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
        P.uncertainty_gamma, P.uncertainty_gamma_min, P.normalize_uncertainty, P.inf_thresh,
        None if P.num_masks <= 0 else P.num_masks, P.force_unmatched_class_to_background,
        P.force_unmatched_masks_to_empty, P.topk_matches, strat, P.mask_gamma,
        None if P.mask_alpha < 0 else P.mask_alpha, P.cls_gamma,
        None if P.cls_alpha < 0 else P.cls_alpha,
        None if P.void_class_index < 0 else P.void_class_index,
        "softmax" if P.use_softmax_label_loss else "sigmoid")
    np.testing.assert_array_equal(p2g.cpu().numpy(), d["pred_to_gt"])
    np.testing.assert_array_equal(prd.cpu().numpy(), d["pred_round"])
    close(m.detach().cpu().numpy(), d["layer_mask_mean"], what="mask mean")
    close(dd.detach().cpu().numpy(), d["layer_dice_mean"], what="dice mean")
    close(c.detach().cpu().numpy(), d["layer_cls_mean"], what="cls mean")
    a = torch.from_numpy(d["upstream"]).to(DEV).float()
    (a[0] * m + a[1] * dd + a[2] * c).sum().backward()
    close_grad(ml.grad.cpu().numpy(), d["grad_mask_logits"], "grad mask")
    close_grad(cl.grad.cpu().numpy(), d["grad_cls_logits"], "grad cls")


@pytest.mark.parametrize("name", case_names())
def test_golden_binding_backward_without_saved_stats(name):
    """The binding-compatible backward recomputes the statistics itself."""
    d, P = load(name)
    ml, mt, cl, ct = to_dev(d)
    p2g = torch.from_numpy(d["pred_to_gt"]).to(DEV)
    a = torch.from_numpy(d["upstream"]).to(DEV).float().contiguous()
    gm, gc = ops.mask_matching_backward(a[0].contiguous(), a[1].contiguous(), a[2].contiguous(),
                                        ml, mt, cl, ct, p2g, *bwd_args(P))
    close_grad(gm.cpu().numpy(), d["grad_mask_logits"], "grad mask")
    close_grad(gc.cpu().numpy(), d["grad_cls_logits"], "grad cls")


# --------------------------------------------------------------------------
# solver: bit-exact on identical fp64 matrices
# --------------------------------------------------------------------------
def test_solver_reference_fixtures_bit_exact():
    s = np.load(GOLDEN + "/solver.npz")
    for c, meta, p2g, prd in zip(s["costs"], s["meta"], s["pred_to_gt"], s["pred_round"]):
        Q, G, strat, K, thr = int(meta[0]), int(meta[1]), int(meta[2]), int(meta[3]), meta[4]
        cd = torch.from_numpy(np.ascontiguousarray(c[:Q, :G])).to(DEV)
        a, r = ops.match_costs(cd, thr, K, strat)
        np.testing.assert_array_equal(a.cpu().numpy(), p2g[:Q], err_msg=str(meta))
        np.testing.assert_array_equal(r.cpu().numpy(), prd[:Q], err_msg=str(meta))


@pytest.mark.parametrize("strategy", [0, 1, 2, 3])
def test_solver_random_bit_exact(strategy):
    rng = np.random.default_rng(11 + strategy)
    for Q, G in [(100, 15), (200, 200), (64, 100), (37, 5), (300, 120), (1100, 12)]:
        for K in (1, 2, 3):
            c = rng.random((3, Q, G))
            c[rng.random(c.shape) < 0.05] = np.inf
            if K == 2:
                c = np.round(c * 8) / 8  # exact ties
            cd = torch.from_numpy(c).to(DEV)
            a, r = ops.match_costs(cd, 1e30, K, strategy)
            for i in range(3):
                ea, er = O.assign_slice(c[i], 1e30, K, strategy)
                np.testing.assert_array_equal(a[i].cpu().numpy(), ea, err_msg=f"{Q}x{G} K={K}")
                np.testing.assert_array_equal(r[i].cpu().numpy(), er, err_msg=f"{Q}x{G} K={K}")
    ops.check_status(block=True)


def test_solver_heavy_ties_signed_zero_bit_exact():
    # costs from a 4-value set (most Dijkstra steps meet equal minima), some
    # of them -0.0 and negative, every strategy, register and shared paths
    rng = np.random.default_rng(23)
    for Q, G in [(20, 7), (50, 30), (100, 21), (127, 60), (260, 40)]:
        c = rng.integers(-1, 3, (2, Q, G)).astype(np.float64) * 0.25
        c[c == 0.0] = np.where(rng.random(int((c == 0.0).sum())) < 0.5, -0.0, 0.0)
        cd = torch.from_numpy(c).to(DEV)
        for strategy in range(4):
            for K in (1, 2):
                a, r = ops.match_costs(cd, 1e30, K, strategy)
                for i in range(2):
                    ea, er = O.assign_slice(c[i], 1e30, K, strategy)
                    np.testing.assert_array_equal(a[i].cpu().numpy(), ea, err_msg=f"{Q}x{G} s={strategy} K={K}")
                    np.testing.assert_array_equal(r[i].cpu().numpy(), er, err_msg=f"{Q}x{G} s={strategy} K={K}")
    ops.check_status(block=True)


def test_solver_fp32_costs_equal_fp64_of_same_values():
    rng = np.random.default_rng(5)
    c32 = rng.random((4, 100, 30)).astype(np.float32)
    a32, r32 = ops.match_costs(torch.from_numpy(c32).to(DEV))
    a64, r64 = ops.match_costs(torch.from_numpy(c32.astype(np.float64)).to(DEV))
    assert torch.equal(a32, a64) and torch.equal(r32, r64)


def test_solver_edge_cases():
    # all-inf column, G > Q, K = 0, NaN entries
    c = np.random.default_rng(1).random((2, 6, 9))
    c[0, :, 2] = np.inf
    c[1, 1, :] = np.nan
    cd = torch.from_numpy(c).to(DEV)
    for K in (0, 1, 2):
        for s in range(4):
            a, r = ops.match_costs(cd, 1e30, K, s)
            for i in range(2):
                ea, er = O.assign_slice(c[i], 1e30, K, s)
                np.testing.assert_array_equal(a[i].cpu().numpy(), ea)
                np.testing.assert_array_equal(r[i].cpu().numpy(), er)
    ops.check_status(block=True)


# --------------------------------------------------------------------------
# generated cases against the oracle
# --------------------------------------------------------------------------
def run_case(batch, kw):
    ml = batch["mask_logits"].to(DEV).contiguous()
    mt = batch["mask_targets"].to(DEV).contiguous()
    cl = batch["cls_logits"].to(DEV).contiguous()
    ct = batch["cls_targets"].to(DEV).contiguous()
    return ml, mt, cl, ct


def oracle_params(kw) -> O.Params:
    return O.Params(**{k: v for k, v in kw.items()})


@pytest.mark.parametrize("ug", [0.0, 1.0])
def test_cfg1_against_oracle(ug):
    cfg = synthetic.CONFIGS["cfg1"]
    batch = synthetic.make_batch(cfg)
    kw = synthetic.parity_kwargs(cfg, uncertainty_gamma=ug)
    ml, mt, cl, ct = run_case(batch, kw)
    P = oracle_params(kw)
    p2g, prd, means, saved, costs = ops.mask_matching_ex(ml, mt, cl, ct, *op_args(P),
                                                         want_saved=True, want_costs=True)
    x, t, z, y = (batch[k].numpy() for k in ("mask_logits", "mask_targets", "cls_logits", "cls_targets"))
    ep2g, eprd, em, ed, ec, esep = O.mask_matching(x, t, z, y, P)
    close(costs.cpu().numpy(), esep, what="costs")
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    np.testing.assert_array_equal(prd.cpu().numpy(), eprd)
    close(means.cpu().numpy(), np.stack([em, ed, ec]), what="means")
    g = torch.tensor([[1.0], [0.7], [1.3]], device=DEV)
    gm, gc = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(), g[2].contiguous(), ml, mt,
                                        cl, ct, p2g, *bwd_args(P), saved=saved)
    egm, egc = O.mask_matching_backward([1.0], [0.7], [1.3], x, t, z, y, ep2g, P)
    close_grad(gm.cpu().numpy(), egm, "grad mask")
    close_grad(gc.cpu().numpy(), egc, "grad cls")


@pytest.mark.parametrize("variant", ["s4_unc", "s2_focal_forced", "sigmoid_round_k2"])
def test_strided_targets_against_oracle(variant):
    torch.manual_seed(3)
    L, B, Q, H, W = 2, 2, 24, 16, 20
    s = {"s4_unc": 4, "s2_focal_forced": 2, "sigmoid_round_k2": 1}[variant]
    C = 9
    ml = torch.randn(L, B, Q, H, W) * 3
    cfg = synthetic.Config("t", 9, L, B, Q, H, W, s, C, 3.0, "ellipse", ("fixed", 6), (0.01, 0.2))
    labs = [synthetic.make_image_labels(cfg, b)[0] for b in range(B)]
    mt = torch.from_numpy(np.stack(labs))
    G = 7
    ct = torch.randint(0, C - 1, (B, G))
    ct[:, 0] = -1
    cl = torch.randn(L, B, Q, C)
    kw = dict(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
              uncertainty_gamma=0.0, uncertainty_gamma_min=0.05, inf_thresh=1e30, num_masks=-1.0,
              force_unmatched_class_to_background=True, force_unmatched_masks_to_empty=False,
              topk_matches=1, strategy_id=0, mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0,
              cls_alpha=-1.0, void_class_index=C - 1, use_softmax_label_loss=True,
              normalize_uncertainty=True)
    if variant == "s4_unc":
        kw.update(uncertainty_gamma=1.0, num_masks=5.0)
    elif variant == "s2_focal_forced":
        kw.update(mask_gamma=2.0, mask_alpha=0.25, force_unmatched_masks_to_empty=True, topk_matches=2)
    else:
        kw.update(use_softmax_label_loss=False, cls_gamma=1.5, cls_alpha=0.3, strategy_id=1,
                  topk_matches=2, normalize_uncertainty=False, uncertainty_gamma=0.5)
    P = oracle_params(kw)
    d = [v.to(DEV).contiguous() for v in (ml, mt, cl, ct)]
    p2g, prd, means, saved, costs = ops.mask_matching_ex(*d, *op_args(P), want_saved=True,
                                                         want_costs=True)
    ep2g, eprd, em, ed, ec, esep = O.mask_matching(ml.numpy(), mt.numpy(), cl.numpy(), ct.numpy(), P)
    close(costs.cpu().numpy(), esep, what="costs")
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    np.testing.assert_array_equal(prd.cpu().numpy(), eprd)
    close(means.cpu().numpy(), np.stack([em, ed, ec]), what="means")
    g = torch.tensor([[0.9, 1.1], [0.5, 1.5], [1.0, 2.0]], device=DEV)
    for sv in (saved, None):
        gm, gc = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(), g[2].contiguous(),
                                            *d[:4], p2g, *bwd_args(P), saved=sv)
        egm, egc = O.mask_matching_backward([0.9, 1.1], [0.5, 1.5], [1.0, 2.0], ml.numpy(),
                                            mt.numpy(), cl.numpy(), ct.numpy(), ep2g, P)
        close_grad(gm.cpu().numpy(), egm, "grad mask")
        close_grad(gc.cpu().numpy(), egc, "grad cls")


@pytest.mark.parametrize("ug", [0.0, 1.0])
def test_wide_mixed_cells_against_oracle(ug):
    # uniform random labels at s = 4: most cells hold more than four output
    # columns, so the mixed-cell table marks them wide and the kernels count
    # those cells from the label map; the rest go through the table
    torch.manual_seed(11)
    L, B, Q, H, W, s, C = 1, 2, 12, 8, 12, 4, 7
    ml = torch.randn(L, B, Q, H, W) * 3
    mt = torch.randint(-1, 11, (B, H * s, W * s))
    mt[:, : 2 * s, : 2 * s] = 3            # a pure block
    mt[:, 2 * s:3 * s, :] = mt[:, 2 * s:3 * s, :] % 3   # at most three labels per cell
    G = 11
    ct = torch.randint(0, C - 1, (B, G))
    ct[:, 0] = -1
    cl = torch.randn(L, B, Q, C)
    P = O.Params(background_index=0, uncertainty_gamma=ug, num_masks=-1.0, void_class_index=C - 1,
                 use_softmax_label_loss=True, force_unmatched_class_to_background=True)
    d = [v.to(DEV).contiguous() for v in (ml, mt, cl, ct)]
    p2g, prd, means, saved, costs, fws = ops.mask_matching_ex(
        *d, *op_args(P), want_saved=True, want_costs=True, want_workspace=True)
    ep2g, eprd, em, ed, ec, esep = O.mask_matching(ml.numpy(), mt.numpy(), cl.numpy(), ct.numpy(), P)
    close(costs.cpu().numpy(), esep, what="costs")
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    close(means.cpu().numpy(), np.stack([em, ed, ec]), what="means")
    g = torch.tensor([[1.2], [0.8], [1.0]], device=DEV)
    egm, egc = O.mask_matching_backward([1.2], [0.8], [1.0], ml.numpy(), mt.numpy(),
                                        cl.numpy(), ct.numpy(), ep2g, P)
    got = []
    for sv, fw in ((saved, None), (None, None), (saved, fws)):
        gm, gc = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(), g[2].contiguous(),
                                            *d[:4], p2g, *bwd_args(P), saved=sv,
                                            forward_workspace=fw)
        close_grad(gm.cpu().numpy(), egm, "grad mask")
        close_grad(gc.cpu().numpy(), egc, "grad cls")
        got.append(gm)
    # the forward's codes give the same gradient, bit for bit
    assert torch.equal(got[0], got[2])


def test_label_ops_against_oracle():
    torch.manual_seed(0)
    L, B, Q, C, G = 2, 3, 17, 40, 9
    z = torch.randn(L, B, Q, C)
    y = torch.randint(-1, C + 2, (B, G))
    P = O.Params(background_index=2, cls_scale=1.7)
    for softmax in (True, False):
        if softmax:
            got = ops.forward_pw_softmax_label_loss(z.to(DEV), y.to(DEV), 2, 1.7)
            ref = O.pairwise_label_cost(z.numpy(), y.numpy(), P, use_softmax=True)
        else:
            got = ops.forward_pw_sigmoid_label_loss(z.to(DEV), y.to(DEV), 2, 1.7, 2.0, 0.25)
            ref = O.pairwise_label_cost(z.numpy(), y.numpy(), P, use_softmax=False, gamma=2.0,
                                        alpha=0.25)
        close(got.cpu().numpy(), ref, what=f"softmax={softmax}")


def test_standalone_pairwise_mask_ops_against_oracle():
    torch.manual_seed(1)
    L, B, Q, H, W, s = 1, 2, 10, 12, 12, 2
    x = torch.randn(L, B, Q, H, W) * 2
    t = torch.randint(0, 5, (B, H * s, W * s))
    gt_total = int(t.max()) + 1
    P = O.Params(background_index=0, sigmoid_scale=3.0, dice_scale=3.0, uncertainty_gamma=1.0)
    ref = O.pairwise_mask_cost(x.numpy(), t.numpy(), gt_total, P)
    sce = ops.forward_pw_sigmoid_ce_loss(x.to(DEV), t.to(DEV), 0, 3.0, 0.0, -1.0, 1.0, 0.05, True)
    dice = ops.forward_pw_dice_loss(x.to(DEV), t.to(DEV), 1.0, 0, 3.0, 1.0, 0.05)
    close(sce.cpu().numpy(), ref[0], what="sigmoid-ce")
    close(dice.cpu().numpy(), ref[1], what="dice")
    # with the GT count passed in (no host read of the targets): the same values
    sce2 = ops.forward_pw_sigmoid_ce_loss(x.to(DEV), t.to(DEV), 0, 3.0, 0.0, -1.0, 1.0, 0.05, True,
                                          num_gts=gt_total)
    dice2 = ops.forward_pw_dice_loss(x.to(DEV), t.to(DEV), 1.0, 0, 3.0, 1.0, 0.05, num_gts=gt_total)
    assert torch.equal(sce2, sce) and torch.equal(dice2, dice)


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("s", [1, 4])
def test_half_logits_equal_fp32_path_on_widened_values(dt, s):
    # 16-bit mask logits: the kernels widen each value exactly and then run
    # the fp32 arithmetic, so costs, assignment and losses equal the fp32 path
    # on the widened tensor bit for bit, and the gradient equals its fp32
    # gradient rounded to the same type; the fp32 path is pinned to the oracle
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16}[dt]
    torch.manual_seed(5 + s)
    L, B, Q, H, W, C = 2, 2, 40, 24, 32, 9
    cfg = synthetic.Config("t", 9, L, B, Q, H, W, s, C, 3.0, "ellipse", ("fixed", 6), (0.01, 0.2))
    mt = torch.from_numpy(np.stack([synthetic.make_image_labels(cfg, b)[0] for b in range(B)]))
    ct = torch.randint(0, C - 1, (B, 7))
    ct[:, 0] = -1
    x16 = (torch.randn(L, B, Q, H, W) * 3).to(dtype)
    cl = torch.randn(L, B, Q, C)
    for ug in (0.0, 1.0):
        P = O.Params(background_index=0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                     uncertainty_gamma=ug, void_class_index=C - 1, use_softmax_label_loss=True,
                     force_unmatched_class_to_background=True)
        d16 = [v.to(DEV).contiguous() for v in (x16, mt, cl, ct)]
        d32 = [d16[0].float()] + d16[1:]
        r16 = ops.mask_matching_ex(*d16, *op_args(P), want_saved=True, want_costs=True)
        r32 = ops.mask_matching_ex(*d32, *op_args(P), want_saved=True, want_costs=True)
        for a, b, what in zip(r16, r32, ("pred_to_gt", "pred_round", "means", "saved", "costs")):
            assert torch.equal(a, b), what
        ep2g, _, em, ed, ec, esep = O.mask_matching(x16.float().numpy(), mt.numpy(), cl.numpy(),
                                                    ct.numpy(), P)
        close(r32[4].cpu().numpy(), esep, what="costs")
        np.testing.assert_array_equal(r32[0].cpu().numpy(), ep2g)
        g = torch.tensor([[0.9, 1.1], [0.5, 1.5], [1.0, 2.0]], device=DEV)
        for sv in (r16[3], None):
            gm16, gc16 = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(),
                                                    g[2].contiguous(), *d16, r16[0], *bwd_args(P),
                                                    saved=sv)
            gm32, gc32 = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(),
                                                    g[2].contiguous(), *d32, r32[0], *bwd_args(P),
                                                    saved=sv)
            assert gm16.dtype == dtype
            assert torch.equal(gm16, gm32.to(dtype))
            assert torch.equal(gc16, gc32)


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_half_logits_through_the_function(dt):
    # autograd: the gradient of 16-bit mask logits arrives in their type and
    # equals the fp32 gradient of the widened logits, rounded
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16}[dt]
    cfg = synthetic.CONFIGS["cfg1"]
    batch = synthetic.make_batch(cfg)
    kw = synthetic.parity_kwargs(cfg)
    ml = batch["mask_logits"].to(DEV).to(dtype)
    mt, cl, ct = (batch[k].to(DEV) for k in ("mask_targets", "cls_logits", "cls_targets"))
    x = ml.clone().requires_grad_(True)
    z = cl.clone().requires_grad_(True)
    p2g, prd, m, d, c = F.MaskMatchingFunction.apply(
        x, mt, z, ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
        kw["background_index"], 0.0, 0.05, True, kw["inf_thresh"], -1.0, True, False, 1, "global",
        0.0, None, None, None, kw["void_class_index"], "softmax")
    (m + d + c).sum().backward()
    assert x.grad.dtype == dtype and torch.isfinite(x.grad.float()).all()
    x32 = ml.float().clone().requires_grad_(True)
    z32 = cl.clone().requires_grad_(True)
    o32 = F.MaskMatchingFunction.apply(
        x32, mt, z32, ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
        kw["background_index"], 0.0, 0.05, True, kw["inf_thresh"], -1.0, True, False, 1, "global",
        0.0, None, None, None, kw["void_class_index"], "softmax")
    (o32[2] + o32[3] + o32[4]).sum().backward()
    assert torch.equal(p2g, o32[0])
    assert torch.equal(x.grad, x32.grad.to(dtype))


def test_odd_query_count_with_plain_load_producer():
    # Q = 129: two query tiles of 65 rows, the second one row past Q; H*W = 35
    # is not a multiple of 16 bytes in either type, so the cost kernel's
    # producer uses plain loads (rows past Q read as zeros)
    torch.manual_seed(129)
    L, B, Q, H, W, s, C = 1, 2, 129, 5, 7, 2, 6
    cfg = synthetic.Config("t", 9, L, B, Q, H, W, s, C, 3.0, "ellipse", ("fixed", 5), (0.05, 0.4))
    mt = torch.from_numpy(np.stack([synthetic.make_image_labels(cfg, b)[0] for b in range(B)]))
    ct = torch.randint(0, C - 1, (B, 6))
    ct[:, 0] = -1
    ml = torch.randn(L, B, Q, H, W) * 3
    cl = torch.randn(L, B, Q, C)
    P = O.Params(background_index=0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0,
                 uncertainty_gamma=0.0, void_class_index=C - 1, use_softmax_label_loss=True,
                 force_unmatched_class_to_background=True)
    d = [v.to(DEV).contiguous() for v in (ml, mt, cl, ct)]
    p2g, prd, means, saved, costs = ops.mask_matching_ex(*d, *op_args(P), want_saved=True,
                                                         want_costs=True)
    ep2g, eprd, em, ed, ec, esep = O.mask_matching(ml.numpy(), mt.numpy(), cl.numpy(), ct.numpy(), P)
    close(costs.cpu().numpy(), esep, what="costs")
    np.testing.assert_array_equal(p2g.cpu().numpy(), ep2g)
    close(means.cpu().numpy(), np.stack([em, ed, ec]), what="means")
    g = torch.tensor([[1.0], [0.6], [1.4]], device=DEV)
    gm, gc = ops.mask_matching_backward(g[0].contiguous(), g[1].contiguous(), g[2].contiguous(),
                                        *d, p2g, *bwd_args(P), saved=saved)
    egm, egc = O.mask_matching_backward([1.0], [0.6], [1.4], ml.numpy(), mt.numpy(), cl.numpy(),
                                        ct.numpy(), ep2g, P)
    close_grad(gm.cpu().numpy(), egm, "grad mask")
    close_grad(gc.cpu().numpy(), egc, "grad cls")
    # the same through 16-bit logits: equal to fp32 on the widened values
    d16 = [d[0].to(torch.bfloat16)] + d[1:]
    d32 = [d16[0].float()] + d[1:]
    r16 = ops.mask_matching_ex(*d16, *op_args(P), want_saved=True, want_costs=True)
    r32 = ops.mask_matching_ex(*d32, *op_args(P), want_saved=True, want_costs=True)
    for a, b in zip(r16, r32):
        assert torch.equal(a, b)


def test_reference_benchmark_shape_properties():
    """The reference harness's mask_matching shape (benchmarks.py:550-614): ten
    decoder layers, 8 images, Q=128, 256x256 logits against 1024x1024 label
    maps, C=128, bg=0, num_masks=5, forced unmatched class, void = C-1,
    softmax label loss, K=1 global.  Size-independent checks only."""
    base = synthetic.CONFIGS["native"]
    cfg = synthetic.Config("ref-bench", base.cfg, 10, base.B, base.Q, base.H, base.W, base.s, base.C,
                           base.logit_std, base.shapes, base.g_law, base.area)
    batch = synthetic.make_batch(cfg, device=DEV, logits=False)
    mt, ct = batch["mask_targets"].contiguous(), batch["cls_targets"].contiguous()
    g = torch.Generator(device=DEV).manual_seed(550)
    ml = torch.randn((cfg.L, cfg.B, cfg.Q, cfg.H, cfg.W), generator=g, device=DEV)
    cl = torch.randn((cfg.L, cfg.B, cfg.Q, cfg.C), generator=g, device=DEV)
    kw = synthetic.parity_kwargs(cfg)
    kw["num_masks"] = 5.0
    P = oracle_params(kw)
    p2g, prd, means, saved, costs = ops.mask_matching_ex(ml, mt, cl, ct, *op_args(P),
                                                         want_saved=True, want_costs=True)
    again = ops.mask_matching_ex(ml, mt, cl, ct, *op_args(P), want_saved=True, want_costs=True)
    assert torch.equal(p2g, again[0]) and torch.equal(costs, again[4])
    assert torch.isfinite(means).all()
    G = ct.shape[1]
    counts = torch.stack([torch.bincount(mt[b].flatten(), minlength=G)[:G] for b in range(cfg.B)])[:, 1:]
    absent = (counts == 0)[None, :, None, :].expand(cfg.L, cfg.B, cfg.Q, -1)
    assert torch.equal(torch.isinf(costs[0]), absent)
    for l in range(cfg.L):
        for b in range(cfg.B):
            m = p2g[l, b][p2g[l, b] >= 0]
            assert torch.equal(torch.sort(m).values, torch.nonzero(~absent[l, b, 0]).flatten())
    tot = (costs[0] + costs[1]) + costs[2]
    for l, b in ((0, 0), (4, 3), (9, 7)):
        ea, _ = O.assign_slice(tot[l, b].double().cpu().numpy(), 1e30, 1, 0)
        np.testing.assert_array_equal(p2g[l, b].cpu().numpy(), ea)
    up = torch.ones(cfg.L, device=DEV)
    gm, gc = ops.mask_matching_backward(up, up, up, ml, mt, cl, ct, p2g, *bwd_args(P), saved=saved)
    assert torch.isfinite(gm).all() and torch.isfinite(gc).all()
    # the mask gradient reaches matched rows only (no forced-empty masks)
    rows = gm.abs().flatten(3).amax(3)
    assert torch.equal(rows[p2g < 0], torch.zeros_like(rows[p2g < 0]))
    assert (rows[p2g >= 0] > 0).all()


def test_deterministic_runs():
    cfg = synthetic.CONFIGS["cfg1"]
    batch = synthetic.make_batch(cfg)
    kw = synthetic.parity_kwargs(cfg, 1.0)
    d = run_case(batch, kw)
    P = oracle_params(kw)
    r1 = ops.mask_matching_ex(*d, *op_args(P), want_saved=True, want_costs=True)
    r2 = ops.mask_matching_ex(*d, *op_args(P), want_saved=True, want_costs=True)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)


def test_cfg2_full_size_properties():
    """Size-independent checks at the Mask2Former COCO shape."""
    cfg = synthetic.CONFIGS["cfg2"]
    batch = synthetic.make_batch(cfg, device=DEV)
    kw = synthetic.parity_kwargs(cfg)
    P = oracle_params(kw)
    ml, mt, cl, ct = (batch[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                      "cls_targets"))
    p2g, prd, means, saved, costs = ops.mask_matching_ex(ml, mt, cl, ct, *op_args(P),
                                                         want_saved=True, want_costs=True)
    again = ops.mask_matching_ex(ml, mt, cl, ct, *op_args(P), want_saved=True, want_costs=True)
    assert torch.equal(p2g, again[0]) and torch.equal(costs, again[4])
    # +inf exactly where a GT id paints no pixel
    counts = torch.stack([torch.bincount(mt[b].flatten(), minlength=ct.shape[1])[:ct.shape[1]]
                          for b in range(cfg.B)])[:, 1:]
    absent = (counts == 0)[None, :, None, :].expand(1, cfg.B, cfg.Q, -1)
    assert torch.equal(torch.isinf(costs[0]), absent)
    # every present GT is matched exactly once (K=1, Q >= G)
    for b in range(cfg.B):
        m = p2g[0, b][p2g[0, b] >= 0]
        assert torch.equal(torch.sort(m).values, torch.nonzero(~absent[0, b, 0]).flatten())
    # the assignment is optimal against the fp64 oracle solver on the same costs
    tot = (costs[0] + costs[1]) + costs[2]
    for b in (0, 7, 15):
        ea, er = O.assign_slice(tot[0, b].double().cpu().numpy(), 1e30, 1, 0)
        np.testing.assert_array_equal(p2g[0, b].cpu().numpy(), ea)
    # layer means equal the gather of matched costs plus the unmatched class terms
    mm = p2g[0] >= 0
    g = p2g[0].clamp(min=0)[..., None]
    sel = torch.gather(costs[:, 0], 3, g[None].expand(3, -1, -1, -1))[..., 0]
    nm = mm.sum().float()
    np.testing.assert_allclose(means[0, 0].item(), (sel[0][mm].sum() / nm).item(), rtol=1e-4)
    np.testing.assert_allclose(means[1, 0].item(), (sel[1][mm].sum() / nm).item(), rtol=1e-4)
