"""The dense-mask oracle reduces to the label-map oracle on non-overlapping
masks (the pinned definition it extends)."""
import numpy as np

from mask_loss_b200 import synthetic
from oracle import dense as D
from oracle import oracle as O


def test_dense_oracle_equals_label_oracle_without_overlap():
    cfg = synthetic.CONFIGS["cfg1"]
    b = synthetic.make_batch(cfg)
    mt = b["mask_targets"].numpy()
    ct = b["cls_targets"].numpy()
    GT = ct.shape[1]
    masks = np.stack([(mt == g) for g in range(GT)], 1).astype(np.uint8)
    P = O.Params(**synthetic.parity_kwargs(cfg))
    ml, cl = b["mask_logits"].numpy(), b["cls_logits"].numpy()
    a = O.mask_matching(ml, mt, cl, ct, P)
    d = D.mask_matching(ml, masks, cl, ct, P)
    np.testing.assert_allclose(d[5], a[5], rtol=1e-12)
    np.testing.assert_array_equal(d[0], a[0])
    for u, v in zip(d[2:5], a[2:5]):
        np.testing.assert_allclose(u, v, rtol=1e-12)
    L = ml.shape[0]
    g = np.linspace(0.5, 1.5, L)
    ga = O.mask_matching_backward(g, g, g, ml, mt, cl, ct, a[0], P)
    gd = D.mask_matching_backward(g, g, g, ml, masks, cl, ct, d[0], P)
    np.testing.assert_allclose(gd[0], ga[0], rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(gd[1], ga[1], rtol=1e-12, atol=1e-15)
