"""Packed variable-length batches and token-superposition (TST) bag batches
against fixtures produced by the reference's own PackedTokenizedCollator
(main.py:57-129), build_token_superposition_batch (:243-352) and
bag_label_entropy_floor (:187-215) (tests/golden/gen_golden.py, gen_data):
every output tensor bit-identical, same dtypes.  Plus properties the formats
guarantee (cu_seqlens / unpad_indices consistency, no bag crossing a segment
boundary) on larger seeded inputs."""
import numpy as np
import pytest
import torch

from zs_b200.data import (PackedTokenizedCollator, bag_label_entropy_floor, build_token_superposition_batch,
                          bucket_max_seqlen, ce_equivalent_reducible_loss, sample_superposition_size)


def _examples(g):
    lens = g["lens"]
    toks = g["tokens"].astype(np.int64)
    out, off = [], 0
    for n in lens:
        out.append({"token_ids": [int(t) for t in toks[off:off + n]]})
        off += n
    return out


def _check(out, g, keys):
    for k in keys:
        ref = g[k]
        got = out[k]
        if torch.is_tensor(got):
            assert str(got.dtype).split(".")[-1] == {"int64": "int64", "int32": "int32", "bool": "bool"}[str(ref.dtype)], k
            got = got.numpy()
        assert np.array_equal(np.asarray(got), ref), k


@pytest.mark.parametrize("name", ["pack_a", "pack_b"])
def test_packed_collator_matches_reference(golden, name):
    g = golden(name)
    out = PackedTokenizedCollator(int(g["L"]), 0)(_examples(g))
    _check(out, g, ["input_ids", "attention_mask", "loss_mask", "position_ids", "cu_seqlens", "unpad_indices",
                    "max_seqlen"])


@pytest.mark.parametrize("name", ["tst_a_pack_a", "tst_a_pack_b", "tst_b_pack_b"])
def test_token_superposition_batch_matches_reference(golden, name):
    t = golden(name)
    g = golden(str(t["src"]))
    packed = PackedTokenizedCollator(int(g["L"]), 0)(_examples(g))
    out = build_token_superposition_batch(packed, int(t["s_bag"]), int(t["latent"]), 0)
    _check(out, t, ["input_ids", "attention_mask", "position_ids", "cu_seqlens", "unpad_indices", "max_seqlen",
                    "loss_indices", "labels", "s"])
    floor = bag_label_entropy_floor(out["labels"], out["s"])
    assert np.array_equal(floor.numpy(), t["floor"])


def test_packed_batch_properties():
    g = np.random.default_rng(4)
    L = 512
    ex = [{"token_ids": list(g.integers(1, 50000, size=int(n)))} for n in g.integers(0, 700, size=300)]
    out = PackedTokenizedCollator(L, 0)(ex)
    cu, unpad = out["cu_seqlens"].long(), out["unpad_indices"]
    assert cu[-1] == unpad.numel() == int(out["attention_mask"].sum())
    # every unpadded position is live, in order, and position ids restart per segment
    assert bool(out["attention_mask"].view(-1)[unpad].all())
    assert bool((unpad[1:] > unpad[:-1]).all())
    pos = out["position_ids"].view(-1)[unpad]
    starts = cu[:-1]
    assert bool((pos[starts] == 0).all())
    assert int((~out["loss_mask"] & out["attention_mask"]).sum()) == cu.numel() - 1
    toks = torch.tensor([t for e in ex for t in e["token_ids"][:L]], dtype=torch.long)
    assert torch.equal(out["input_ids"].view(-1)[unpad], toks)
    # TST: bags never straddle a segment, labels are the next bag of the same segment
    tb = build_token_superposition_batch(out, 4, 96, 0)
    bags = tb["input_ids"].view(-1, 4)[tb["unpad_indices"]]
    seg_lens = (tb["cu_seqlens"][1:] - tb["cu_seqlens"][:-1]).tolist()
    off, lab_off = 0, 0
    for n in seg_lens:
        assert torch.equal(tb["labels"][lab_off:lab_off + n - 1], bags[off + 1:off + n])
        off, lab_off = off + n, lab_off + n - 1
    assert tb["labels"].size(0) == tb["loss_indices"].numel() == tb["s"].numel()


def test_small_helpers():
    assert bucket_max_seqlen(0, 4096) == 0 and bucket_max_seqlen(33, 4096) == 64 and bucket_max_seqlen(5000, 4096) == 4096
    assert sample_superposition_size(0.05, 4) == 4 and sample_superposition_size(0.5, 4) == 1
    assert sample_superposition_size(0.0, 1) == 1
    raw = torch.tensor(5.0)
    loss, gap = ce_equivalent_reducible_loss(raw, 65536, torch.tensor(1.0))
    lv = float(np.log(65536))
    assert abs(float(loss) - (5.0 - 1.0) * lv / (lv - 1.0)) < 1e-5 and abs(float(gap) - (lv - 1.0)) < 1e-5
    assert build_token_superposition_batch({"input_ids": torch.zeros(1, 8, dtype=torch.long),
                                            "cu_seqlens": torch.tensor([0, 5], dtype=torch.int32),
                                            "unpad_indices": torch.arange(5)}, 4, 16, 0) is None
    with pytest.raises(ValueError):
        build_token_superposition_batch({}, 1, 16, 0)
