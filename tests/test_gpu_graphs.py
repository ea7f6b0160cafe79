"""MatchingLossStep: a CUDA-graph replay of matching + loss forward/backward
gives the eager results, and follows new data written into its inputs."""
import pytest
import torch

from mask_loss_b200 import synthetic
from mask_loss_b200 import functions as F
from mask_loss_b200.graphs import MatchingLossStep

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _args(cfg):
    kw = synthetic.parity_kwargs(cfg, uncertainty_gamma=1.0)
    return [kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
            kw["background_index"], kw["uncertainty_gamma"], kw["uncertainty_gamma_min"], True,
            kw["inf_thresh"], None, True, False, 1, "global", 0.0, None, None, None,
            kw["void_class_index"], "softmax"]


def _eager(ml, mt, cl, ct, args):
    x = ml.clone().requires_grad_(True)
    z = cl.clone().requires_grad_(True)
    p2g, prd, m, d, c = F.MaskMatchingFunction.apply(x, mt, z, ct, *args)
    (m + d + c).sum().backward()
    return p2g, torch.stack([m, d, c]).detach(), x.grad, z.grad


def test_graph_replay_matches_eager_and_tracks_inputs():
    cfg = synthetic.CONFIGS["cfg1"]
    b = synthetic.make_batch(cfg, device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    args = _args(cfg)
    step = MatchingLossStep(ml.clone(), mt.clone(), cl.clone(), ct.clone(), *args)
    for scale in (1.0, 0.5):
        step.inputs["mask_logits"].copy_(ml * scale)
        step.replay()
        torch.cuda.synchronize()
        step.check()
        p2g, losses, gm, gc = _eager(ml * scale, mt, cl, ct, args)
        assert torch.equal(step.pred_to_gt, p2g)
        torch.testing.assert_close(step.losses, losses, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(step.grad_mask_logits, gm, rtol=1e-5, atol=1e-9)
        torch.testing.assert_close(step.grad_cls_logits, gc, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_graph_replay_with_16bit_mask_logits(dtype):
    # 4x label map so the backward reuses the forward's cell codes
    cfg = synthetic.CONFIGS["cfg3"]
    b = synthetic.make_batch(cfg, images=[0, 1], device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    ml = ml.to(dtype)
    args = _args(cfg)
    step = MatchingLossStep(ml.clone(), mt.clone(), cl.clone(), ct.clone(), *args)
    step.replay()
    torch.cuda.synchronize()
    step.check()
    p2g, losses, gm, gc = _eager(ml, mt, cl, ct, args)
    assert step.grad_mask_logits.dtype == dtype
    assert torch.equal(step.pred_to_gt, p2g)
    torch.testing.assert_close(step.losses, losses, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(step.grad_mask_logits, gm, rtol=0, atol=0)
    torch.testing.assert_close(step.grad_cls_logits, gc, rtol=1e-5, atol=1e-9)


def test_auto_num_masks_counts_present_gts():
    cfg = synthetic.CONFIGS["cfg1"]
    b = synthetic.make_batch(cfg, device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    args = _args(cfg)
    present = sum(int((torch.unique(mt[i]) > 0).sum()) for i in range(cfg.B))
    a_auto = list(args); a_auto[9] = "auto"
    a_num = list(args); a_num[9] = float(present)
    r1 = _eager(ml, mt, cl, ct, a_auto)
    r2 = _eager(ml, mt, cl, ct, a_num)
    # force_unmatched_class=True makes the class term use B*Q; mask/dice use num_masks
    for x, y in zip(r1[1:], r2[1:]):
        torch.testing.assert_close(x, y, rtol=1e-6, atol=1e-9)


def test_void_class_in_targets_raises_deferred():
    """functions/mask/matching.py:180-181: a void id in cls_targets is an
    error of the Function (checked on the device, raised without a host
    sync) and of the graph step; the binding-level op does not check."""
    from mask_loss_b200 import ops
    cfg = synthetic.CONFIGS["cfg1"]
    b = synthetic.make_batch(cfg, device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    args = _args(cfg)
    bad = ct.clone()
    bad[0, 1] = args[18]  # a GT column labelled with the void class
    ops.check_status(block=True)
    F.MaskMatchingFunction.apply(ml, mt, cl, bad, *args)
    with pytest.raises(RuntimeError, match="void class index"):
        ops.check_status(block=True)
    F.MaskMatchingFunction.apply(ml, mt, cl, ct, *args)
    ops.check_status(block=True)  # clean targets: nothing pending
    kw = synthetic.parity_kwargs(cfg)
    ops.mask_matching(ml, mt, cl, bad, *list(kw.values()))
    ops.check_status(block=True)  # the binding op has no such check
    step = MatchingLossStep(ml.clone(), mt.clone(), cl.clone(), ct.clone(), *args)
    step.replay()
    step.check()
    step.inputs["cls_targets"].copy_(bad)
    step.replay()
    with pytest.raises(RuntimeError, match="void class index"):
        step.check()


@pytest.mark.parametrize("opt", ["zero_fill_beside_solver"])
@pytest.mark.parametrize("cname,dtype", [("cfg1", torch.float32), ("cfg3", torch.bfloat16)])
def test_graph_step_with_the_gradient_zeroed_early(opt, cname, dtype):
    # the mask gradient zeroed on a side stream beside the solver and then
    # written only on the rows the loss reaches: the
    # same results as the default step, bit for bit, over replays whose
    # matched rows change (the buffer keeps no stale rows)
    cfg = synthetic.CONFIGS[cname]
    b = synthetic.make_batch(cfg, images=[0, 1], device=DEV)
    ml, mt, cl, ct = (b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                                  "cls_targets"))
    ml = ml.to(dtype)
    args = _args(cfg)
    ref = MatchingLossStep(ml.clone(), mt.clone(), cl.clone(), ct.clone(), *args)
    alt = MatchingLossStep(ml.clone(), mt.clone(), cl.clone(), ct.clone(), *args, **{opt: True})
    for scale in (1.0, -0.7):
        for s in (ref, alt):
            s.inputs["mask_logits"].copy_(ml * scale)
            s.replay()
        torch.cuda.synchronize()
        ref.check()
        alt.check()
        assert torch.equal(alt.pred_to_gt, ref.pred_to_gt)
        assert torch.equal(alt.losses, ref.losses)
        assert torch.equal(alt.grad_mask_logits, ref.grad_mask_logits)
        assert torch.equal(alt.grad_cls_logits, ref.grad_cls_logits)
