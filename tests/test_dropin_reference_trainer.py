"""The drop-in boundary seen from the reference's own trainer: with this package's
import root in front of a reference checkout, the reference's main.py imports
unchanged; its own modeling/model.py builds the model from this package's
modules (attention, MoE layer, experts, norms), and its optimizer and
checkpoint helpers come from this package (the reference's other helpers, e.g. utils/tokenizer.py, stay
reachable).  Runs in a subprocess; skipped where no reference checkout exists
(the GPU box has none).  No GPU work: the model and optimizer are only built."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "architecture-zarelga-superposition_b200"
REF = Path(os.environ.get("ZS_REFERENCE", "/root/reference"))

SCRIPT = r"""
import torch
import main
from modeling.model_config import ModelConfig

pkg = {pkg!r}
cfg = ModelConfig(vocab_size=128, embed_size=64, hidden_size=64, transformer_depth=2, intermediate_size=32,
                  n_experts=5, n_shared_experts=1, n_experts_per_token=2, n_attention_heads=2, n_key_value_heads=1,
                  attention_window_pattern=(None, None), max_position_embeddings=64, sequence_length=64,
                  pos_rope_dims=8)
model = main.MoEModel(cfg)
opt = main.build_muonmd_optimizer(model, torch.device("cpu"))
where = {{
    "MoEModel": type(model).__init__.__code__.co_filename,
    "GLUMLP": type(model.layers[0].mlp.routed_experts).forward.__code__.co_filename,
    "attention": type(model.layers[0].self_attn).forward.__code__.co_filename,
    "dense_optimizer": type(opt.dense).__init__.__code__.co_filename,
    "hybrid": type(opt).__init__.__code__.co_filename,
    "sparse_optimizer": type(opt.sparse).__init__.__code__.co_filename,
    "save_checkpoint": main.save_checkpoint.__code__.co_filename,
    "linear_cross_entropy": main.linear_cross_entropy.__code__.co_filename,
    "mcce": main.mcce_raw_token_mean_v2.__code__.co_filename,
    "zRMSNorm": main.ZeroCenteredRMSNorm.__init__.__code__.co_filename,
}}
# the reference's own model.py builds the model, on this package's modules
assert where.pop("MoEModel").startswith({ref!r}), type(model)
bad = {{k: v for k, v in where.items() if not v.startswith(pkg)}}
assert not bad, bad
import utils.tokenizer  # the reference's own helper, still importable
assert not utils.tokenizer.__file__.startswith(pkg)
# the reference's packed collator output drives this package's data helpers unchanged
batch = main.PackedTokenizedCollator(32, 0)([{{"token_ids": list(range(1, 20))}}, {{"token_ids": list(range(5, 30))}}])
from zs_b200.data import PackedTokenizedCollator
mine = PackedTokenizedCollator(32, 0)([{{"token_ids": list(range(1, 20))}}, {{"token_ids": list(range(5, 30))}}])
assert all(torch.equal(batch[k], mine[k]) if torch.is_tensor(batch[k]) else batch[k] == mine[k] for k in batch)
print("ok", len(where))
"""


@pytest.mark.skipif(not (REF / "main.py").exists(), reason="no reference checkout on this machine")
def test_reference_trainer_imports_and_builds_on_this_package(tmp_path):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(PKG), str(REF)])
    env["PYTHONDONTWRITEBYTECODE"] = "1"
    # aim (the reference's metrics logger) is absent here; main.py only imports its name
    stub = tmp_path / "stubs"
    stub.mkdir()
    (stub / "aim.py").write_text("Distribution = Run = None\n")
    env["PYTHONPATH"] = os.pathsep.join([env["PYTHONPATH"], str(stub)])
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(pkg=str(PKG), ref=str(REF))], cwd=tmp_path, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.strip().startswith("ok")
