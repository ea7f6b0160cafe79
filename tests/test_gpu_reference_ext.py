"""This library against the reference's own CUDA extension, at the one shape
the reference dispatches (src/cuda/pw_mask.cu:377-382: Q=128, 256x256 logits,
1024x1024 label maps, C=128) -- the harness of benchmarks.py:550-614.

The extension is built from the reference sources by
``oracle/build_ref_ext.py`` into oracle/_ref/ext; without it these tests are
skipped.  Its ops are called directly with the binding's 24 / 25 positional
arguments (src/bindings.cpp:86-139), since the reference's Python wrapper
passes 25 arguments to the 24-argument forward binding
(functions/mask/matching.py:198-224).

Parity (L=1, tie-free images): identical assignments, layer means within
1e-4 relative, both gradients within 1e-4 relative / 1e-5 of the largest
magnitude.  With ten layers the costs and layer means are compared (the
random logits are not tie-filtered per layer).  Both tests print the
forward + backward time of each implementation (CUDA events, after warm-up).
"""
import glob
import importlib.util
import os

import numpy as np
import pytest
import torch

from fullsize import DEV, Case
from mask_loss_b200 import functions as F
from mask_loss_b200 import ops, synthetic
from mask_loss_b200.graphs import MatchingLossStep
from oracle import oracle as O

pytestmark = pytest.mark.gpu

EXT = sorted(glob.glob(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "oracle", "_ref", "ext", "mask_loss*.so")))


def ref_ext():
    if not EXT:
        pytest.skip("reference extension not built (oracle/build_ref_ext.py)")
    spec = importlib.util.spec_from_file_location("mask_loss", EXT[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def harness_cfg(L):
    base = synthetic.CONFIGS["native"]
    return synthetic.Config(f"native-l{L}", base.cfg, L, base.B, base.Q, base.H, base.W, base.s,
                            base.C, base.logit_std, base.shapes, base.g_law, base.area)


def harness_params(cfg):
    # benchmarks.py:550-614: uncertainty weights on, num_masks=5, unmatched
    # queries to the void class C-1, softmax label loss, K=1 global
    kw = synthetic.parity_kwargs(cfg, uncertainty_gamma=1.0)
    kw["num_masks"] = 5.0
    return O.Params(**kw)


def fwd_args(P):
    return (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
            P.uncertainty_gamma, P.uncertainty_gamma_min, P.inf_thresh, P.num_masks,
            P.force_unmatched_class_to_background, P.force_unmatched_masks_to_empty,
            P.topk_matches, P.strategy_id, P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha,
            P.void_class_index, P.use_softmax_label_loss, P.normalize_uncertainty)


def bwd_args(P):
    return (P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale, P.background_index,
            P.uncertainty_gamma, P.uncertainty_gamma_min, P.num_masks,
            P.force_unmatched_class_to_background, P.force_unmatched_masks_to_empty,
            P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha, P.void_class_index,
            P.use_softmax_label_loss, P.normalize_uncertainty)


def timed_ms(fn, n=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def run_both(ref, d, P):
    L = d[0].shape[0]
    up = [torch.full((L,), v, device=DEV) for v in (1.0, 0.7, 1.3)]

    def reference():
        p2g, prd, m, dd, c = ref.mask_matching(*d, *fwd_args(P))
        gm, gc = ref.mask_matching_backward(*up, *d, p2g, *bwd_args(P))
        return p2g, prd, torch.stack([m, dd, c]), gm, gc

    def ours():
        x = d[0].detach().requires_grad_(True)
        z = d[2].detach().requires_grad_(True)
        p2g, prd, m, dd, c = F.MaskMatchingFunction.apply(
            x, d[1], z, d[3], P.smooth, P.sigmoid_scale, P.dice_scale, P.cls_scale,
            P.background_index, P.uncertainty_gamma, P.uncertainty_gamma_min,
            P.normalize_uncertainty, P.inf_thresh, P.num_masks,
            P.force_unmatched_class_to_background, P.force_unmatched_masks_to_empty,
            P.topk_matches, "global", P.mask_gamma, None, None, None, P.void_class_index,
            "softmax")
        (up[0] * m + up[1] * dd + up[2] * c).sum().backward()
        return p2g, prd, torch.stack([m, dd, c]).detach(), x.grad, z.grad

    return reference, ours, up


def report(tag, ref_fn, our_fn, graph):
    t_ref = timed_ms(ref_fn)
    t_ours = timed_ms(our_fn)
    t_graph = timed_ms(graph.replay)
    print(f"\nREFERENCE-EXTENSION {tag}: reference fwd+bwd {t_ref:.3f} ms, this library "
          f"autograd fwd+bwd {t_ours:.3f} ms ({t_ref / t_ours:.1f}x), graph step "
          f"{t_graph:.3f} ms ({t_ref / t_graph:.1f}x)")


def graph_step(d, P, L):
    g = MatchingLossStep(*[t.clone() for t in d], P.smooth, P.sigmoid_scale, P.dice_scale,
                         P.cls_scale, P.background_index, P.uncertainty_gamma,
                         P.uncertainty_gamma_min, True, P.inf_thresh, P.num_masks,
                         P.force_unmatched_class_to_background,
                         P.force_unmatched_masks_to_empty, 1, "global", 0.0, None, None, None,
                         P.void_class_index, "softmax", loss_weights=(1.0, 0.7, 1.3))
    return g


def test_reference_extension_one_layer():
    ref = ref_ext()
    cfg = harness_cfg(1)
    P = harness_params(cfg)
    case = Case(cfg, range(cfg.B), P)
    d = [case.batch[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits",
                                               "cls_targets")]
    reference, ours, _ = run_both(ref, d, P)
    rp2g, rprd, rmeans, rgm, rgc = reference()
    op2g, oprd, omeans, ogm, ogc = ours()
    assert torch.equal(rp2g, op2g), "assignments differ from the reference extension"
    assert torch.equal(rprd, oprd)
    np.testing.assert_allclose(omeans.cpu().numpy(), rmeans.cpu().numpy(), rtol=1e-4, atol=1e-5)
    for got, exp, what in ((ogm, rgm, "grad mask"), (ogc, rgc, "grad cls")):
        e = exp.double().cpu().numpy()
        np.testing.assert_allclose(got.double().cpu().numpy(), e, rtol=1e-4,
                                   atol=1e-5 * np.abs(e).max(), err_msg=what)
    # and both against the CPU oracle's assignment
    ep2g, _, _, _ = case.oracle_forward()
    np.testing.assert_array_equal(op2g.cpu().numpy(), ep2g)
    report("L=1 (8 x Q=128 x 256^2, labels 1024^2)", reference, ours, graph_step(d, P, 1))
    ops.check_status(block=True)


def test_reference_extension_ten_layers():
    ref = ref_ext()
    cfg = harness_cfg(10)
    P = harness_params(cfg)
    b = synthetic.make_batch(cfg, device=DEV)
    d = [b[k].contiguous() for k in ("mask_logits", "mask_targets", "cls_logits", "cls_targets")]
    rc = ref.pairwise_mask_loss_forward(d[0], d[1], d[2], d[3], P.smooth, P.sigmoid_scale,
                                        P.dice_scale, P.cls_scale, P.background_index,
                                        P.uncertainty_gamma, P.uncertainty_gamma_min,
                                        P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha,
                                        P.use_softmax_label_loss, P.normalize_uncertainty)
    oc = ops.pairwise_mask_loss_forward(d[0], d[1], d[2], d[3], P.smooth, P.sigmoid_scale,
                                        P.dice_scale, P.cls_scale, P.background_index,
                                        P.uncertainty_gamma, P.uncertainty_gamma_min,
                                        P.mask_gamma, P.mask_alpha, P.cls_gamma, P.cls_alpha,
                                        P.use_softmax_label_loss, P.normalize_uncertainty)
    r, o = rc.double().cpu().numpy(), oc.double().cpu().numpy()
    assert np.array_equal(np.isinf(r), np.isinf(o))
    f = np.isfinite(r)
    np.testing.assert_allclose(o[f], r[f], rtol=1e-4, atol=1e-5)
    reference, ours, _ = run_both(ref, d, P)
    rp2g, _, rmeans, _, _ = reference()
    op2g, _, omeans, _, _ = ours()
    same = (rp2g == op2g).float().mean().item()
    assert same > 0.99, f"only {same:.4f} of the assignments agree"
    np.testing.assert_allclose(omeans.cpu().numpy(), rmeans.cpu().numpy(), rtol=1e-4, atol=1e-5)
    report("L=10 (the harness shape)", reference, ours, graph_step(d, P, 10))
    ops.check_status(block=True)
