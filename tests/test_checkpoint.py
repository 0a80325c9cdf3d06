"""Checkpoint format (utils/trainutils.py:34-88): a checkpoint written by the
reference's save_checkpoint after one step of its optimizer
(tests/golden/gen_golden.py, gen_ckpt) loads into this package's MoEModel and
optimizer (strict state dict, optimizer state intact); this package's
checkpoints have the reference's tensor names, shapes and dtypes and round-trip
exactly; on the GPU, the optimizer state written after a real step has the
reference's per-parameter layout (keys, shapes, dtypes)."""
import shutil

import pytest
import torch

from _util import GOLDEN_DIR

CKPT_CONFIG = dict(vocab_size=128, embed_size=32, hidden_size=32, transformer_depth=2, intermediate_size=16,
                   n_experts=5, n_shared_experts=1, n_experts_per_token=2, n_attention_heads=2, n_key_value_heads=1,
                   attention_window_pattern=(None, None), max_position_embeddings=32, sequence_length=32,
                   pos_rope_dims=8)


def _model_opt(device="cpu"):
    from zs_b200.lm import MoELM as MoEModel
    from modeling.model_config import ModelConfig
    from zs_b200.train import build_muonmd_optimizer

    torch.manual_seed(0)
    model = MoEModel(ModelConfig(**CKPT_CONFIG)).to(device)
    return model, build_muonmd_optimizer(model, torch.device(device))


def _state_equal(a, b):
    if torch.is_tensor(a):
        return torch.is_tensor(b) and a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.cpu(), b.cpu())
    if isinstance(a, dict):
        return isinstance(b, dict) and a.keys() == b.keys() and all(_state_equal(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)):
        return len(a) == len(b) and all(_state_equal(x, y) for x, y in zip(a, b))
    return a == b


def test_reference_checkpoint_loads(tmp_path):
    from safetensors.torch import load_file
    from utils.trainutils import load_checkpoint

    src = GOLDEN_DIR / "ckpt_ref.safetensors"
    shutil.copy(src, tmp_path / "c.safetensors")
    shutil.copy(GOLDEN_DIR / "ckpt_ref.trainer.pt", tmp_path / "c.trainer.pt")
    model, opt = _model_opt()
    meta = load_checkpoint(model, opt, str(tmp_path / "c.safetensors"))
    assert meta == {"global_step": 1, "epoch": 0}
    ref = load_file(str(src))
    mine = model.state_dict()
    assert set(ref) == set(mine)
    for k, v in ref.items():
        assert torch.equal(mine[k], v), k
    trainer = torch.load(GOLDEN_DIR / "ckpt_ref.trainer.pt", weights_only=False)
    assert _state_equal(opt.state_dict()["dense"]["state"], trainer["optimizer"]["dense"]["state"])
    assert _state_equal(opt.state_dict()["sparse"]["state"], trainer["optimizer"]["sparse"]["state"])
    assert opt.state_dict()["dense_steps"] == trainer["optimizer"]["dense_steps"]


def test_checkpoint_names_shapes_and_round_trip(tmp_path):
    from safetensors import safe_open
    from utils.trainutils import load_checkpoint, save_checkpoint

    model, opt = _model_opt()
    with torch.no_grad():
        for p in model.parameters():
            p.add_(torch.randn_like(p) * 0.01)
    save_checkpoint(model, opt, str(tmp_path / "m.safetensors"), global_step=7, epoch=2)

    def layout(path):
        with safe_open(str(path), "pt") as f:
            return {k: (tuple(f.get_slice(k).get_shape()), f.get_slice(k).get_dtype()) for k in f.keys()}

    assert layout(tmp_path / "m.safetensors") == layout(GOLDEN_DIR / "ckpt_ref.safetensors")
    model2, opt2 = _model_opt()
    assert load_checkpoint(model2, opt2, str(tmp_path / "m.safetensors")) == {"global_step": 7, "epoch": 2}
    for (k, a), (_, b) in zip(model.state_dict().items(), model2.state_dict().items()):
        assert torch.equal(a, b), k


def _layout(state):
    return {pid: {k: (tuple(v.shape), v.dtype) if torch.is_tensor(v) else type(v).__name__ for k, v in st.items()}
            for pid, st in state.items()}


@pytest.mark.gpu
def test_optimizer_state_layout_after_a_gpu_step_matches_reference(tmp_path):
    from utils.trainutils import save_checkpoint

    model, opt = _model_opt("cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    emb = model.embedding.weight
    for p in model.parameters():
        if p is emb:
            rows = torch.tensor([[1, 5, 9, 77]], device="cuda")
            p.grad = torch.sparse_coo_tensor(rows, torch.randn(4, p.size(1), device="cuda", generator=g), p.shape)
        else:
            p.grad = torch.randn(p.shape, device="cuda", generator=g) * 0.01
    opt.step()
    torch.cuda.synchronize()
    save_checkpoint(model, opt, str(tmp_path / "g.safetensors"), global_step=1, epoch=0)
    mine = torch.load(tmp_path / "g.trainer.pt", map_location="cpu", weights_only=False)["optimizer"]
    ref = torch.load(GOLDEN_DIR / "ckpt_ref.trainer.pt", weights_only=False)["optimizer"]
    assert _layout(mine["dense"]["state"]) == _layout(ref["dense"]["state"])
    assert _layout(mine["sparse"]["state"]) == _layout(ref["sparse"]["state"])
    assert [len(g_["params"]) for g_ in mine["dense"]["param_groups"]] == \
        [len(g_["params"]) for g_ in ref["dense"]["param_groups"]]
