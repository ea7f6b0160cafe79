"""GPU parity of the standalone semantic losses (sigmoid CE, dice) against
the reference's fixtures and the CPU oracle; tolerances as elsewhere:
losses 1e-4 relative, gradients 1e-5 of the tensor's largest magnitude."""
import glob
import os

import numpy as np
import pytest
import torch

from mask_loss_b200 import functions as F
from mask_loss_b200 import ops
from oracle import semantic as S

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "semantic_*.npz")))


def close_grad(got, ref):
    ref = np.asarray(ref, np.float64)
    np.testing.assert_allclose(np.asarray(got, np.float64), ref, rtol=1e-4,
                               atol=1e-5 * max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("name", NAMES)
def test_semantic_golden_functions(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    x = torch.from_numpy(d["logits"]).to(DEV)
    t = torch.from_numpy(d["targets"]).to(DEV)
    go = torch.from_numpy(d["grad_out"]).to(DEV).float()
    nm, sc, ga, al = (float(v) for v in d["sce_kw"])
    xs = x.clone().requires_grad_(True)
    ls = F.SigmoidCELossFunction.apply(xs, t, nm, sc, ga, None if al < 0 else al)
    (ls * go).sum().backward()
    np.testing.assert_allclose(ls.detach().cpu().numpy(), d["sce_loss"], rtol=1e-4)
    close_grad(xs.grad.cpu().numpy(), d["sce_grad"])
    sm, nm, sc = (float(v) for v in d["dice_kw"])
    xd = x.clone().requires_grad_(True)
    ld = F.DiceLossFunction.apply(xd, t, sm, nm, sc)
    (ld * go).sum().backward()
    np.testing.assert_allclose(ld.detach().cpu().numpy(), d["dice_loss"], rtol=1e-4)
    close_grad(xd.grad.cpu().numpy(), d["dice_grad"])


def _random_case(seed, L, B, C, H, W, s, noisy):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(L, B, C, H, W, generator=g) * 2.5
    if noisy:  # per-pixel labels: many cells with more than four labels, some out of range
        t = torch.randint(-1, C + 1, (B, H * s, W * s), generator=g)
    else:
        t = torch.randint(0, C, (B, H, W), generator=g).repeat_interleave(s, 1).repeat_interleave(s, 2)
    go = torch.rand(L, generator=g) + 0.5
    return x, t, go


@pytest.mark.parametrize("case", [
    (1, 2, 3, 9, 13, 1, False), (2, 1, 7, 16, 16, 4, True), (1, 3, 20, 8, 8, 2, True),
    (3, 2, 133, 16, 16, 1, False), (1, 1, 5, 17, 19, 3, True),
    (1, 2, 300, 9, 7, 5, True), (2, 1, 11, 6, 5, 6, False)])
def test_semantic_random_against_oracle(case):
    x, t, go = _random_case(sum(case[:6]), *case)
    xd_, td_, god = x.to(DEV), t.to(DEV), go.to(DEV)
    for gamma, alpha in ((0.0, -1.0), (2.0, 0.25), (1.5, -1.0)):
        out = ops.forward_sigmoid_ce_loss(xd_, td_, 4.0, 1.3, gamma, alpha)
        gr = ops.backward_sigmoid_ce_loss(god, xd_, td_, 4.0, 1.3, gamma, alpha)
        el, eg = S.sigmoid_ce(x.numpy(), t.numpy(), 4.0, 1.3, gamma, alpha, grad_out=go.numpy())
        np.testing.assert_allclose(out.cpu().numpy(), el, rtol=1e-4)
        close_grad(gr.cpu().numpy(), eg)
    out, I, P, T = ops.forward_dice_loss(xd_, td_, 1.0, 6.0, 0.8)
    gr = ops.backward_dice_loss(god, xd_, td_, I, P, T, 1.0, 6.0, 0.8)
    el, eI, eP, eT, eg = S.dice(x.numpy(), t.numpy(), 1.0, 6.0, 0.8, grad_out=go.numpy())
    np.testing.assert_allclose(out.cpu().numpy(), el, rtol=1e-4)
    np.testing.assert_allclose(I.cpu().numpy(), eI, rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(P.cpu().numpy(), eP, rtol=1e-4, atol=1e-3)
    np.testing.assert_array_equal(T.cpu().numpy(), eT)
    close_grad(gr.cpu().numpy(), eg)


def test_semantic_deterministic_and_edges():
    x, t, go = _random_case(5, 2, 2, 9, 12, 12, 2, True)
    xd_, td_ = x.to(DEV), t.to(DEV)
    a = ops.forward_sigmoid_ce_loss(xd_, td_, 3.0)
    b = ops.forward_sigmoid_ce_loss(xd_, td_, 3.0)
    assert torch.equal(a, b)
    a = ops.forward_dice_loss(xd_, td_, 1.0, 3.0)
    b = ops.forward_dice_loss(xd_, td_, 1.0, 3.0)
    assert all(torch.equal(u, v) for u, v in zip(a, b))
    # empty class axis: zero losses, as the reference returns
    e = torch.zeros(2, 2, 0, 12, 12, device=DEV)
    assert torch.equal(ops.forward_sigmoid_ce_loss(e, td_, 1.0), torch.zeros(2, device=DEV))
    assert torch.equal(ops.forward_dice_loss(e, td_, 1.0, 1.0)[0], torch.zeros(2, device=DEV))
    with pytest.raises(RuntimeError, match="integer multiple"):
        ops.forward_sigmoid_ce_loss(xd_, td_[:, :23].contiguous(), 1.0)


@pytest.mark.parametrize("four_d", [False, True])
def test_losses_front_end_equals_the_functions(four_d):
    # functions/losses.py:8-67 with class_mapping=None: the same values and
    # gradients as the Functions it wraps, for (L,B,C,h,w) and (B,C,h,w) logits
    x, t, go = _random_case(17, 2, 2, 6, 12, 12, 2, False)
    x, t = x.to(DEV), t.to(DEV)
    if four_d:
        x = x[0]
    for front, fn, extra in ((F.sigmoid_cross_entropy_loss, F.SigmoidCELossFunction, ()),
                             (F.dice_loss, F.DiceLossFunction, (1e-6,))):
        xa = x.clone().requires_grad_(True)
        xb = x.clone().requires_grad_(True)
        la = front(xa, t, *extra, num_masks=7.0, scale=1.5)
        lb = fn.apply(xb[None] if four_d else xb, t, *extra, 7.0, 1.5)
        lb = lb[0] if four_d else lb
        assert la.shape == lb.shape
        la.sum().backward()
        lb.sum().backward()
        assert torch.equal(la.detach(), lb.detach())
        assert torch.equal(xa.grad, xb.grad)
