"""The reference's own Python wrappers run against this package's op surface.

``mask_loss_b200.ops`` is meant to stand in for the reference extension
module (``sys.modules["mask_loss"] = mask_loss_b200.ops``, src/bindings.cpp:
157-169).  Here the reference's ``functions`` package is imported with a
recording stand-in for ``mask_loss`` whose every op first binds the wrapper's
arguments to the signature of the same-named op in ``mask_loss_b200.ops`` --
so a call that the B200 op would reject for its arity or argument names fails
here the same way -- and then answers with the CPU oracle (the hot pairwise
op) or zeros of the op's output shape, so the wrapper can finish.

CPU only (no kernels run); skipped when the reference checkout is not found
(``MASK_LOSS_REF`` or a ``reference`` directory beside the repository): it is
never present on the GPU box.
"""
import contextlib
import importlib
import inspect
import io
import sys
import types

import numpy as np
import pytest
import torch

from mask_loss_b200 import ops
from oracle import oracle as O

REF = O.reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not found")


class Recorder:
    def __init__(self):
        self.calls = []


def _gt_out(gt_total, bg):
    return gt_total - (1 if 0 <= bg < gt_total else 0)


def _shim(rec: Recorder) -> types.ModuleType:
    m = types.ModuleType("mask_loss")

    def op(name, out):
        sig = inspect.signature(getattr(ops, name))

        def f(*args):
            sig.bind(*args)  # TypeError on an arity or order mismatch, as the B200 op would
            rec.calls.append(name)
            return out(*args)
        setattr(m, name, f)

    def pairwise(ml, mt, cl, ct, smooth, ss, ds, cs, bg, ug, ugmin, mg, ma, cg, ca, sm, norm):
        P = O.Params(smooth=smooth, sigmoid_scale=ss, dice_scale=ds, cls_scale=cs,
                     background_index=bg, uncertainty_gamma=ug, uncertainty_gamma_min=ugmin,
                     mask_gamma=mg, mask_alpha=ma, cls_gamma=cg, cls_alpha=ca,
                     use_softmax_label_loss=sm, normalize_uncertainty=norm)
        return torch.from_numpy(O.pairwise_mask_loss(ml.numpy(), mt.numpy(), cl.numpy(),
                                                     ct.numpy(), P).astype(np.float32))

    def pw_mask_only(logits, targets, *rest):
        bg = rest[0] if isinstance(rest[0], int) else rest[1]
        g = int(targets.max()) + 1
        L, B, Q = logits.shape[:3]
        return torch.zeros(L, B, Q, _gt_out(g, bg))

    def pw_label(logits, targets, bg, *rest):
        L, B, Q = logits.shape[:3]
        return torch.zeros(L, B, Q, _gt_out(targets.shape[1], bg))

    op("pairwise_mask_loss_forward", pairwise)
    op("forward_pw_sigmoid_ce_loss", pw_mask_only)
    op("forward_pw_dice_loss", pw_mask_only)
    op("forward_pw_sigmoid_label_loss", pw_label)
    op("forward_pw_softmax_label_loss", pw_label)
    op("forward_sigmoid_ce_loss", lambda x, *r: torch.zeros(x.shape[0]))
    op("backward_sigmoid_ce_loss", lambda g, x, *r: torch.zeros_like(x))
    op("forward_dice_loss", lambda x, *r: [torch.zeros(x.shape[0])] +
       [torch.zeros(x.shape[:3]) for _ in range(3)])
    op("backward_dice_loss", lambda g, x, *r: torch.zeros_like(x))
    op("mask_matching", lambda ml, *r: [torch.zeros(ml.shape[:3], dtype=torch.int64)] * 2 +
       [torch.zeros(ml.shape[0])] * 3)
    op("mask_matching_backward", lambda gm, gd, gc, ml, mt, cl, *r: [torch.zeros_like(ml),
                                                                     torch.zeros_like(cl)])
    return m


@pytest.fixture()
def ref_functions():
    rec = Recorder()
    saved = {k: v for k, v in sys.modules.items() if k == "mask_loss" or k == "functions" or
             k.startswith("functions.")}
    for k in saved:
        del sys.modules[k]
    sys.modules["mask_loss"] = _shim(rec)
    sys.path.insert(0, REF)
    try:
        with contextlib.redirect_stdout(io.StringIO()):
            F = importlib.import_module("functions")
        yield F, rec
    finally:
        sys.path.remove(REF)
        for k in [k for k in sys.modules if k == "mask_loss" or k == "functions" or
                  k.startswith("functions.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def _case():
    g = torch.Generator().manual_seed(3)
    L, B, Q, H, W, C, G = 1, 2, 6, 8, 8, 5, 4
    ml = torch.randn(L, B, Q, H, W, generator=g) * 2
    mt = torch.randint(0, G, (B, H * 2, W * 2), generator=g)
    cl = torch.randn(L, B, Q, C, generator=g)
    ct = torch.randint(0, C - 1, (B, G), generator=g)
    ct[:, 0] = -1
    return ml, mt, cl, ct


def test_reference_pairwise_wrappers_reach_the_op_surface(ref_functions):
    F, rec = ref_functions
    ml, mt, cl, ct = _case()
    out = F.PairwiseMaskLossFunction.apply(ml, mt, cl, ct, 1.0, 5.0, 5.0, 2.0, 0, 1.0, 0.05, True,
                                          0.0, None, None, None, "softmax")
    P = O.Params(sigmoid_scale=5.0, dice_scale=5.0, cls_scale=2.0, background_index=0,
                 uncertainty_gamma=1.0, use_softmax_label_loss=True)
    ref = O.pairwise_mask_loss(ml.numpy(), mt.numpy(), cl.numpy(), ct.numpy(), P)
    np.testing.assert_allclose(out.numpy(), ref.astype(np.float32))
    F.PairwiseSigmoidCELossFunction.apply(ml, mt, 0, 1.0, 0.0, None)
    F.PairwiseDiceLossFunction.apply(ml, mt, 1.0, 0, 1.0)
    F.PairwiseSigmoidLabelLossFunction.apply(cl, ct, 0, 1.0, 0.0, None)
    F.PairwiseSoftmaxLabelLossFunction.apply(cl, ct, 0, 1.0)
    assert rec.calls == ["pairwise_mask_loss_forward", "forward_pw_sigmoid_ce_loss",
                         "forward_pw_dice_loss", "forward_pw_sigmoid_label_loss",
                         "forward_pw_softmax_label_loss"]


def test_reference_semantic_wrappers_reach_the_op_surface(ref_functions):
    F, rec = ref_functions
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, 2, 3, 4, 4, generator=g).requires_grad_(True)
    t = torch.randint(0, 3, (2, 8, 8), generator=g)
    F.SigmoidCELossFunction.apply(x, t, 6.0, 1.0, 0.0, None).sum().backward()
    x.grad = None
    F.DiceLossFunction.apply(x, t, 1.0, 6.0).sum().backward()
    assert rec.calls == ["forward_sigmoid_ce_loss", "backward_sigmoid_ce_loss",
                         "forward_dice_loss", "backward_dice_loss"]


def test_reference_matching_wrapper_keeps_its_arity_bug(ref_functions):
    # functions/mask/matching.py:198-224 passes 25 arguments to the 24-argument
    # mask_matching binding (src/bindings.cpp:86-111): the B200 op surface,
    # like the reference's pybind11 module, refuses the call.  This package's
    # own MaskMatchingFunction calls the op with the binding's order.
    F, rec = ref_functions
    ml, mt, cl, ct = _case()
    with pytest.raises(TypeError, match="too many positional arguments"):
        F.MaskMatchingFunction.apply(ml, mt, cl, ct, 1.0, 5.0, 5.0, 2.0, 0, 0.0, 0.05, True, 1e30,
                                     None, True, False, 1, "global", 0.0, None, None, None, 4,
                                     "softmax")
    assert rec.calls == []
