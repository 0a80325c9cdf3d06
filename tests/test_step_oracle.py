"""The whole-step oracle (oracle/model_step.py) against one training step of the
reference itself at BASELINE config 1's shapes (tests/golden/gen_golden.py,
gen_step): the loss, every layer's routing (index sets per token, routing
counts) and gate probabilities, the layer outputs, every parameter's gradient
and its update by the optimizer, and the router biases after the aux-loss-free
update.  Both sides run f32 on the CPU; the Newton-Schulz iterations run in
bf16 on both, so a last-bit difference of a gradient can move an update by a
few tenths of a percent (the update bound below)."""
import numpy as np
import pytest
import torch

from _util import cosine, rel_err
from oracle import model_step as M


@pytest.fixture(scope="module")
def step(golden):
    f = golden("step_cfg1")
    cfg = M.config1()
    P = M.canonical_params(cfg, 0)
    before = {k: v.clone() for k, v in P.items()}
    ids = torch.as_tensor(f["ids"])
    biases = [torch.zeros(cfg["n_routed_experts"]) for _ in range(cfg["transformer_depth"])]
    keep = {}
    torch.manual_seed(0)
    loss, grads, topks = M.train_step(P, {}, biases, cfg, ids, keep=keep)
    return f, cfg, P, before, loss, grads, topks, biases, keep


def test_loss_and_routing(step):
    f, cfg, P, before, loss, grads, topks, biases, keep = step
    assert abs(float(loss) - float(f["loss"])) <= 1e-5 * abs(float(f["loss"]))
    for i, t in enumerate(topks):
        mine = np.sort(t.reshape(-1, cfg["n_experts_per_token"]).numpy(), axis=1)
        ref = np.sort(f[f"topk{i}"].reshape(-1, cfg["n_experts_per_token"]), axis=1)
        assert np.array_equal(mine, ref), f"layer {i} routing"
        assert rel_err(keep[f"layer{i}"]["gate_probs"], f[f"probs{i}"]) < 1e-5
        np.testing.assert_array_equal(biases[i].numpy(), f[f"bias_after{i}"])


def test_layer_outputs(step):
    f, cfg, P, before, loss, grads, topks, biases, keep = step
    for i in range(cfg["transformer_depth"]):
        for key in ("attn", "moe", "out"):
            t = keep[f"layer{i}"][key].reshape(-1)
            assert rel_err(t[torch.as_tensor(f[f"{key}{i}_idx"])], f[f"{key}{i}"]) < 1e-5, (i, key)
            assert abs(float(t.norm()) - float(f[f"{key}{i}_norm"])) <= 1e-5 * float(f[f"{key}{i}_norm"])


def test_gradients_and_updates(step):
    f, cfg, P, before, loss, grads, topks, biases, keep = step
    for name in P:
        idx = torch.as_tensor(f[f"idx:{name}"])
        g = grads[name].reshape(-1)[idx]
        assert rel_err(g, f[f"grad:{name}"]) < 1e-4, name
        assert abs(float(grads[name].norm()) - float(f[f"gnorm:{name}"])) <= 1e-4 * float(f[f"gnorm:{name}"]) + 1e-12
        delta = (P[name] - before[name]).reshape(-1)[idx]
        ref_delta = f[f"delta:{name}"]
        if np.linalg.norm(ref_delta) > 0:
            assert cosine(delta, ref_delta) > 0.999, name
            assert rel_err(delta, ref_delta) < 3e-2, name
        # the bf16 Newton-Schulz turns last-bit gradient differences into ~1.5 % of the
        # orthogonalised update (cosine > 0.9998), ~1e-3 of the weights after the step
        assert rel_err(P[name].reshape(-1)[idx], f[f"after:{name}"]) < 2e-3, name
