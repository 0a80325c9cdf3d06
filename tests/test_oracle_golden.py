"""The CPU oracle against fixtures produced by running the reference itself
(tests/golden/gen_golden.py: the reference's Triton kernels under the Triton
CPU interpreter, MoEGate and flatten_sort_count in CPU PyTorch)."""
import numpy as np
import pytest

from oracle import routing as R
from oracle import scattermoe as S


@pytest.mark.parametrize("case", ["gate_e8_k2", "gate_e64_k8", "gate_e128_k8"])
def test_gate_topk_sets_and_weights(golden, case):
    g = golden(case)
    k = int(g["k"])
    idx, w = R.gate_topk(g["probs"], g["bias"], k, dtype="f32")
    # CPU torch.topk(sorted=False) returns the same set in another order
    ref_idx, ref_w = g["topk_idx"], g["topk_weight"]
    assert np.array_equal(np.sort(idx, 1), np.sort(ref_idx, 1))
    o1, o2 = np.argsort(idx, 1), np.argsort(ref_idx, 1)
    np.testing.assert_allclose(np.take_along_axis(w, o1, 1), np.take_along_axis(ref_w, o2, 1), rtol=2e-6, atol=1e-7)


def test_gate_topk_order_rule():
    # strictly-greater values in index order, then ties at the k-th value in index order
    probs = np.array([[0.5, 0.9, 0.5, 0.7, 0.5, 0.1]], dtype=np.float32)
    idx, _ = R.gate_topk(probs, np.zeros(6, np.float32), 4, dtype="f32")
    assert idx.tolist() == [[1, 3, 0, 2]]


@pytest.mark.parametrize("case", ["fsc_small", "fsc_e64", "fsc_skew"])
def test_flatten_sort_count(golden, case):
    g = golden(case)
    sei, ssi, off = R.flatten_sort_count(g["expert_idxs"], int(g["num_experts"]))
    assert np.array_equal(sei, g["sorted_expert_idxs"])
    assert np.array_equal(off, g["expert_offsets"])
    # The reference's slot order inside an expert's segment is whatever its
    # sort implementation produced (not stable here); the segment's set of
    # flat indices is the contract, and the oracle's order is the stable one.
    start = 0
    for end in off:
        assert np.array_equal(np.sort(ssi[start:end]), np.sort(g["sorted_scattered_idxs"][start:end]))
        assert np.all(np.diff(ssi[start:end]) > 0)
        start = end


def test_scatter2scatter_variants(golden):
    g = golden("ops_f32")
    k = int(g["k"])
    W = np.transpose(g["Wt"], (0, 2, 1))
    sei, ssi = g["sorted_expert_idxs"], g["sorted_scattered_idxs"]
    tol = dict(rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(S.scatter2scatter(g["X"], W, sei, ssi, k, y_grouped=True), g["s2s_xg0_yg1"], **tol)
    np.testing.assert_allclose(S.scatter2scatter(g["X"], W, sei, ssi, k), g["s2s_xg0_yg0"], **tol)
    np.testing.assert_allclose(S.scatter2scatter(g["Xg"], W, sei, ssi, 1, x_grouped=True, y_grouped=True),
                               g["s2s_xg1_yg1"], **tol)
    np.testing.assert_allclose(S.scatter2scatter(g["Xg"], W, sei, ssi, 1, x_grouped=True), g["s2s_xg1_yg0"], **tol)
    np.testing.assert_allclose(S.scatter2scatter(g["DYg"], g["Wt"], sei, ssi, 1, x_grouped=True), g["s2s_wT"], **tol)
    np.testing.assert_allclose(S.scatter2scatter(g["X"], W, sei, ssi, k, b=g["bias"], y_grouped=True), g["s2s_bias"],
                               **tol)


def test_group_xty_group_rsp(golden):
    g = golden("ops_f32")
    k = int(g["k"])
    E = g["Wt"].shape[0]
    np.testing.assert_allclose(S.group_xty(g["DYg"], g["Xg"], g["expert_offsets"], E), g["xty_dw"], rtol=1e-4,
                               atol=1e-4)
    np.testing.assert_allclose(S.group_bias(g["DYg"], g["expert_offsets"], E), g["xty_db"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(S.group(g["X"], g["sorted_scattered_idxs"], k), g["group"], rtol=0, atol=0)
    np.testing.assert_allclose(S.group(g["X"], g["sorted_scattered_idxs"], k, coeff=g["p"]), g["group_coeff"],
                               rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(S.rowwise_sum_product(g["A3"], g["B2"]), g["rsp"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ["glu_small", "glu_e8"])
def test_glu_mlp_forward_backward(golden, case):
    g = golden(case)
    y, saved = S.glu_mlp_forward(g["x"], g["expert_p"], g["expert_idxs"], g["W1"], g["W2"], dtype="f32")
    np.testing.assert_allclose(y, g["y"], rtol=1e-4, atol=1e-5)
    dx, dp, dW1, dW2 = S.glu_mlp_backward(g["dy"], g["x"], g["expert_p"], g["W1"], g["W2"], saved, dtype="f32")
    np.testing.assert_allclose(dx, g["dx"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dp, g["dp"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dW1, g["dW1"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dW2, g["dW2"], rtol=1e-4, atol=1e-5)


def test_aux_loss_free_update_rule():
    topk = np.array([[0, 1], [0, 2], [0, 1]])
    new = R.aux_loss_free_update(np.zeros(4, np.float32), topk, 1e-3)
    # counts [3, 2, 1, 0], mean 1.5
    assert new.tolist() == pytest.approx([-1e-3, -1e-3, 1e-3, 1e-3])
    assert np.array_equal(R.aux_loss_free_update(np.ones(4, np.float32), topk, 1e-3, valid=np.zeros(3, bool)),
                          np.ones(4, np.float32))
