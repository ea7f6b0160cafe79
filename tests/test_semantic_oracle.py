"""The semantic-loss oracle against the reference's own outputs (fixtures
made by tests/golden/make_golden_semantic.py)."""
import glob
import os

import numpy as np
import pytest

from oracle import semantic as S

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "semantic_*.npz")))


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    nm, sc, ga, al = d["sce_kw"]
    loss, grad = S.sigmoid_ce(d["logits"], d["targets"], nm, sc, ga, al, grad_out=d["grad_out"])
    np.testing.assert_allclose(loss, d["sce_loss"], rtol=1e-10)
    np.testing.assert_allclose(grad, d["sce_grad"], rtol=1e-8, atol=1e-14)
    sm, nm, sc = d["dice_kw"]
    loss, I, P, T, grad = S.dice(d["logits"], d["targets"], sm, nm, sc, grad_out=d["grad_out"])
    np.testing.assert_allclose(loss, d["dice_loss"], rtol=1e-10)
    np.testing.assert_allclose(grad, d["dice_grad"], rtol=1e-8, atol=1e-14)


def test_fixtures_present():
    assert len(NAMES) >= 3
