"""The allocation-free cost entry point, called through the C ABI.

Some callers cannot call cudaMalloc -- code running inside a custom
allocator or memory-pool callback, or a process that reserved all device
memory up front -- so ml_pairwise_mask_loss_forward_noalloc keeps its scratch
in a fixed device array inside the library instead of asking for a
workspace.  These checks compare it with the workspace entry point on two
calls in a row (the second call must not see the first call's leftovers in
the shared array) and check that an oversized call is refused.

This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from mask_loss_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
RTOL, ATOL = 1e-4, 1e-5


def _inputs(cfg_name, seed):
    cfg = synthetic.CONFIGS[cfg_name]
    b = synthetic.make_batch(cfg)
    g = torch.Generator().manual_seed(seed)
    ml = (torch.randn(b["mask_logits"].shape, generator=g) * cfg.logit_std).to(DEV)
    return cfg, ml, b["mask_targets"].to(DEV), b["cls_logits"].to(DEV), b["cls_targets"].to(DEV)


def _noalloc(ml, mt, cl, ct, kw):
    lib = _lib.load()
    d = ops._dims(ml, mt, cl, ct)
    p = ops._params(**kw)
    G = lib.ml_gt_out(d.GT_total, p.background_index)
    out = torch.full((3, *ml.shape[:3], G), float("nan"), device=DEV)
    rc = lib.ml_pairwise_mask_loss_forward_noalloc(
        ctypes.byref(d), ctypes.byref(p), ops._ptr(ml), ops._ptr(mt), ops._ptr(cl), ops._ptr(ct),
        ops._ptr(out), ops._stream(ml.device))
    return rc, out


def _with_workspace(ml, mt, cl, ct, kw):
    return ops.pairwise_mask_loss_forward(
        ml, mt, cl, ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
        kw["background_index"], kw["uncertainty_gamma"], kw["uncertainty_gamma_min"],
        kw["mask_gamma"], kw["mask_alpha"], kw["cls_gamma"], kw["cls_alpha"],
        kw["use_softmax_label_loss"], kw["normalize_uncertainty"])


def _close(a, b):
    a = a.cpu().numpy().astype(np.float64)
    b = b.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isinf(a), np.isinf(b))
    f = np.isfinite(b)
    np.testing.assert_allclose(a[f], b[f], rtol=RTOL, atol=ATOL)


def test_noalloc_matches_workspace_entry_on_two_calls():
    # call 1: the Mask2Former COCO shape; call 2: a different, smaller batch;
    # call 3: a 4x label map (codes plus the mixed-cell table in the scratch)
    for cfg_name, seed, ug in (("cfg2", 1, 0.0), ("cfg1", 2, 1.0), ("cfg3", 3, 0.0)):
        cfg, ml, mt, cl, ct = _inputs(cfg_name, seed)
        kw = synthetic.parity_kwargs(cfg, uncertainty_gamma=ug)
        kw.pop("inf_thresh"); kw.pop("num_masks"); kw.pop("force_unmatched_class_to_background")
        kw.pop("force_unmatched_masks_to_empty"); kw.pop("topk_matches"); kw.pop("strategy_id")
        kw.pop("void_class_index")
        rc, got = _noalloc(ml, mt, cl, ct, kw)
        assert rc == 0, _lib.load().ml_last_error()
        ref = _with_workspace(ml, mt, cl, ct, kw)
        torch.cuda.synchronize()
        _close(got, ref)


def test_noalloc_odd_plane_and_no_device_allocation():
    # 33 x 35 cells: H*W is not a multiple of 4, so the cost kernel's producer
    # takes the plain-load path through the shared array; and repeated calls
    # must not take device memory (the driver's free-memory figure stays put;
    # torch's caching allocator is not involved either way)
    torch.manual_seed(7)
    L, B, Q, H, W, C, G = 1, 2, 30, 33, 35, 9, 6
    cfg = synthetic.Config("odd", 9, L, B, Q, H, W, 1, C, 3.0, "ellipse", ("fixed", G - 1),
                           (0.02, 0.3))
    mt = torch.from_numpy(np.stack([synthetic.make_image_labels(cfg, b)[0]
                                    for b in range(B)])).to(DEV)
    ml = (torch.randn(L, B, Q, H, W) * 3).to(DEV)
    cl = torch.randn(L, B, Q, C).to(DEV)
    ct = torch.randint(0, C - 1, (B, G)).to(DEV)
    ct[:, 0] = -1
    kw = dict(smooth=1.0, sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
              uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, mask_gamma=0.0, mask_alpha=-1.0,
              cls_gamma=0.0, cls_alpha=-1.0, use_softmax_label_loss=True,
              normalize_uncertainty=True)
    ref = _with_workspace(ml, mt, cl, ct, kw)
    rc, got = _noalloc(ml, mt, cl, ct, kw)  # first call: any lazy loading happens here
    assert rc == 0, _lib.load().ml_last_error()
    torch.cuda.synchronize()
    _close(got, ref)
    out = torch.empty_like(got)
    lib = _lib.load()
    d = ops._dims(ml, mt, cl, ct)
    p = ops._params(**kw)
    free0 = torch.cuda.mem_get_info(DEV)[0]
    for _ in range(5):
        rc = lib.ml_pairwise_mask_loss_forward_noalloc(
            ctypes.byref(d), ctypes.byref(p), ops._ptr(ml), ops._ptr(mt), ops._ptr(cl),
            ops._ptr(ct), ops._ptr(out), ops._stream(ml.device))
        assert rc == 0
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(DEV)[0]
    assert free1 >= free0, f"device memory dropped by {free0 - free1} bytes"
    _close(out, ref)


def test_noalloc_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    limit = lib.ml_noalloc_scratch_limit()
    assert limit == 64 << 20
    # config-4 shapes (64 images, Q=200, 512x512) need far more scratch; the
    # size check happens before anything is launched, so tiny dummies suffice
    d = _lib.Dims(1, 64, 200, 512, 512, 512, 512, 151, 201)
    p = ops._params(background_index=0, uncertainty_gamma=0.0)
    dummy = torch.zeros(16, device=DEV)
    rc = lib.ml_pairwise_mask_loss_forward_noalloc(
        ctypes.byref(d), ctypes.byref(p), ops._ptr(dummy), ops._ptr(dummy), ops._ptr(dummy),
        ops._ptr(dummy), ops._ptr(dummy), ops._stream(dummy.device))
    assert rc == 6  # ML_EUNSUPPORTED
    assert b"fixed" in lib.ml_last_error()
