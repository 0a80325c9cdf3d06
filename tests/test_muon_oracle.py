"""Newton-Schulz oracle against the reference's own bf16 CPU run."""
import numpy as np

from oracle import muon as M


def _cos(a, b):
    a, b = np.ravel(a), np.ravel(b)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_newton_schulz_oracle(golden):
    g = golden("ns5")
    for G, X in ((g["G_wide"], g["X_wide"]), (g["G_tall"], g["X_tall"])):
        out = M.newton_schulz5(G, 5)
        assert out.shape == X.shape
        assert _cos(out, X) > 0.999
        assert np.linalg.norm(out - X) / np.linalg.norm(X) < 5e-2  # bf16 NS5 chains amplify rounding
