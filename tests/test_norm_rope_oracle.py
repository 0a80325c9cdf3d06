"""zRMSNorm / RoPE oracle against fixtures from the reference (CPU module
autograd; the Liger Triton kernel under the Triton interpreter)."""
import numpy as np
import pytest

from oracle import attention as A


@pytest.mark.parametrize("case", ["zrms_d64", "zrms_d256"])
def test_zrmsnorm_oracle(golden, case):
    g = golden(case)
    y, _ = A.zrmsnorm(g["x"], g["w"], 1e-6)
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)
    dx, dw = A.zrmsnorm_backward(g["dy"], g["x"], g["w"], 1e-6)
    np.testing.assert_allclose(dx, g["dx"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(dw, g["dw"], rtol=1e-4, atol=1e-5)


def test_rope_tables_and_rotation(golden):
    g = golden("rope")
    cos_t, sin_t = A.rope_tables(300, 64, 10000.0, 32)
    np.testing.assert_allclose(cos_t, g["cos_table"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(sin_t, g["sin_table"], rtol=0, atol=2e-6)
    pos = g["pos"]
    cos, sin = g["cos_table"][pos], g["sin_table"][pos]
    np.testing.assert_allclose(A.rope(g["q"], cos, sin), g["q_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(A.rope(g["k"], cos, sin), g["k_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(A.rope(g["dq"], cos, sin, backward=True), g["dq_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(A.rope(g["dk"], cos, sin, backward=True), g["dk_out"], rtol=1e-5, atol=1e-6)
