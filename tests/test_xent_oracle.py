"""The cross-entropy oracle against fixtures from the reference's own CPU
MCCE implementations (naive formulation and autograd; chunked path agrees)."""
import numpy as np
import pytest

from oracle import xent as X


@pytest.mark.parametrize("case", ["mcce_selftest", "mcce_t1", "mcce_t7", "mcce_t33"])
def test_mcce_oracle_matches_reference(golden, case):
    g = golden(case)
    loss, dH, dE = X.mcce(g["hidden"], g["emb"], g["labels"], g["s"])
    np.testing.assert_allclose(loss, g["loss"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dH, g["dH"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(dE, g["dE"], rtol=1e-4, atol=1e-6)


def test_cross_entropy_oracle_matches_torch(golden):
    g = golden("cce_ignore")
    loss, de, dc = X.cross_entropy(g["e"], g["c"], g["targets"])
    np.testing.assert_allclose(loss, g["loss"], rtol=1e-5)
    np.testing.assert_allclose(de, g["de"], rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(dc, g["dc"], rtol=1e-4, atol=1e-7)
