"""Pins the CPU oracle (oracle/oracle.c) to the reference's own outputs.

Fixtures in tests/golden/ were produced by the reference's Python path
(functions/mask/matching.py:336-815) and its compiled C++ solver
(src/cpu/matching.cpp:476-571); see tests/golden/make_golden.py.
"""
import numpy as np
import pytest

from oracle import oracle as O
from golden_cases import case_names, load, GOLDEN

RTOL, ATOL = 1e-6, 1e-8  # oracle (double) vs reference evaluated in float64


@pytest.mark.parametrize("name", case_names())
def test_costs(name):
    d, P = load(name)
    sep = O.pairwise_mask_loss(d["mask_logits"], d["mask_targets"], d["cls_logits"],
                               d["cls_targets"], P)
    ref = d["sep"]
    assert sep.shape == ref.shape
    assert np.array_equal(np.isinf(sep), np.isinf(ref))
    f = np.isfinite(ref)
    np.testing.assert_allclose(sep[f], ref[f], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name", case_names())
def test_matching_and_losses(name):
    d, P = load(name)
    p2g, prd, m, dd, c, _ = O.mask_matching(d["mask_logits"], d["mask_targets"],
                                            d["cls_logits"], d["cls_targets"], P)
    np.testing.assert_array_equal(p2g, d["pred_to_gt"])
    np.testing.assert_array_equal(prd, d["pred_round"])
    np.testing.assert_allclose(m, d["layer_mask_mean"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(dd, d["layer_dice_mean"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(c, d["layer_cls_mean"], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name", case_names())
def test_backward(name):
    d, P = load(name)
    a = d["upstream"]
    gx, gz = O.mask_matching_backward(a[0], a[1], a[2], d["mask_logits"], d["mask_targets"],
                                      d["cls_logits"], d["cls_targets"], d["pred_to_gt"], P)
    np.testing.assert_allclose(gx, d["grad_mask_logits"], rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(gz, d["grad_cls_logits"], rtol=1e-5, atol=1e-9)


def test_solver_matches_reference_fixtures():
    s = np.load(GOLDEN + "/solver.npz")
    for c, meta, p2g, prd in zip(s["costs"], s["meta"], s["pred_to_gt"], s["pred_round"]):
        Q, G, strat, K, thr = int(meta[0]), int(meta[1]), int(meta[2]), int(meta[3]), meta[4]
        a, r = O.assign_slice(c[:Q, :G], thr, K, strat)
        np.testing.assert_array_equal(a, p2g[:Q])
        np.testing.assert_array_equal(r, prd[:Q])


def test_solver_matches_compiled_reference():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    rng = np.random.default_rng(3)
    for _ in range(60):
        Q, G = rng.integers(1, 40), rng.integers(1, 30)
        c = rng.random((Q, G))
        c[rng.random((Q, G)) < 0.15] = np.inf
        if rng.random() < 0.5:
            c = np.round(c * 3) / 3
        for strat in range(4):
            K = int(rng.integers(0, 4))
            a, r = O.assign_slice(c, 1e30, K, strat)
            a2, r2 = O.assign_slice(c, 1e30, K, strat, use_ref=True)
            np.testing.assert_array_equal(a, a2)
            np.testing.assert_array_equal(r, r2)


@pytest.mark.parametrize("name", ["sampled_basic", "sampled_focal_s4", "sampled_align_nobg"])
def test_sampled_costs_against_reference_fixtures(name):
    from oracle import sampled as S
    d = np.load(GOLDEN + f"/{name}.npz")
    Pn, bg, al, fg, fa = d["meta"]
    P = O.Params(background_index=int(bg), sigmoid_scale=2.0, dice_scale=3.0, smooth=1.0,
                 mask_gamma=float(fg), mask_alpha=float(fa))
    gt = int(d["mask_targets"].max()) + 1
    out = S.pairwise_costs_sampled(d["mask_logits"], d["mask_targets"], d["coords"], gt, P,
                                   align_corners=bool(al)).numpy()
    for got, ref in ((out[0], d["sce"]), (out[1], d["dice"])):
        assert np.array_equal(np.isinf(got), np.isinf(ref))
        f = np.isfinite(ref)
        np.testing.assert_allclose(got[f], ref[f], rtol=1e-5, atol=1e-6)
