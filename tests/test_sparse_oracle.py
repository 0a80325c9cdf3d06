"""The sparse-embedding oracle (oracle/sparse.py) against the reference's own
GramReaperSparse run on seeded COO gradients (tests/golden/gen_golden.py,
gen_sparse): duplicate rows, a step that touches nothing, with and without the
unit-norm projection."""
import numpy as np
import pytest

from oracle import sparse as O


@pytest.mark.parametrize("name,unit", [("sparse_unit", True), ("sparse_plain", False)])
def test_sparse_rmsprop_oracle_matches_reference(golden, name, unit):
    f = golden(name)
    p = f["W0"].copy()
    v = np.zeros(p.shape[0], np.float32)
    t = 0
    for k in range(3):
        t = O.sparse_rmsprop_step(p, v, t, f[f"rows{k}"], f[f"vals{k}"], 3e-2, 0.9, 1e-10, unit)
        np.testing.assert_allclose(p, f[f"W{k + 1}"], rtol=2e-6, atol=2e-7)
    np.testing.assert_allclose(v, f["v"], rtol=2e-6, atol=1e-8)
    assert t == int(f["t"]) == 2


def test_embedding_bag_oracle_is_the_lookup_mean():
    rng = np.random.default_rng(3)
    table = rng.standard_normal((30, 8)).astype(np.float32)
    ids = rng.integers(0, 30, size=(2, 5, 3))
    out = O.embedding_bag(table, ids, 2.0)
    ref = table[ids].mean(axis=-2) * 2.0
    np.testing.assert_allclose(out, ref, rtol=1e-6)
    rows, vals = O.embedding_bag_coo(np.ones((2, 5, 8), np.float32), ids, 2.0)
    assert rows.shape == (30,) and vals.shape == (30, 8)
    np.testing.assert_allclose(vals, 2.0 / 3.0, rtol=1e-6)
