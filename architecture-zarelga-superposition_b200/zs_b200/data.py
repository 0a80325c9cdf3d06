"""Input formats of the training step: packed variable-length batches and
token-superposition (TST) bag batches, plus the TST loss rescaling.

Same names, arguments and outputs as the reference trainer's data path
(main.py): TokenizedJsonlDataset (:32-55), PackedTokenizedCollator (:57-129),
bag_label_entropy_floor (:187-215), ce_equivalent_reducible_loss (:217-221),
bucket_max_seqlen (:223-226), sample_superposition_size (:228-240) and
build_token_superposition_batch (:243-352).  The packers build their index
tensors with vectorised numpy/torch (aranges and repeats over segment lengths)
instead of per-token Python loops; the packing decisions are the reference's:
greedy rows in arrival order for the collator, first-fit decreasing (stable
on ties) for TST bags.  The outputs feed GatedAttention / MoELayer's
cu_seqlens / unpad_indices path and the MCCE loss (labels [N, s], s [N]).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import torch


class TokenizedJsonlDataset(torch.utils.data.Dataset):
    """Records (path, byte offset) of pre-tokenized JSONL lines with a `token_ids` field;
    each item is cut to max_length, ending in EOS (one slot reserved when the record
    does not already end in EOS)."""

    def __init__(self, records, max_length, pad_token_id, eos_token_id):
        self.records = records
        self.max_length = max_length
        self.pad_token_id = pad_token_id
        self.eos_token_id = eos_token_id

    def __len__(self):
        return len(self.records)

    def __getitem__(self, idx):
        path, offset = self.records[idx]
        with Path(path).open("rb") as f:
            f.seek(offset)
            ids = json.loads(f.readline().decode("utf-8"))["token_ids"]
        if ids and ids[-1] == self.eos_token_id:
            ids = ids[: self.max_length]
        else:
            ids = ids[: self.max_length - 1] + [self.eos_token_id]
        return {"token_ids": ids}


def bucket_max_seqlen(max_seqlen, max_length):
    if max_seqlen <= 0:
        return 0
    return min(((max_seqlen + 31) // 32) * 32, max_length)


def _segment_layout(lengths, row_of, start_in_row, row_len):
    """Flat (row * row_len + position) index of every token of every segment, the
    position inside its segment, and the segments' inclusive cumulative lengths."""
    lengths = np.asarray(lengths, dtype=np.int64)
    total = int(lengths.sum())
    seg = np.repeat(np.arange(lengths.size), lengths)
    first = np.concatenate([[0], np.cumsum(lengths)[:-1]]) if lengths.size else np.zeros(0, np.int64)
    pos = np.arange(total, dtype=np.int64) - first[seg]
    flat = np.asarray(row_of, np.int64)[seg] * row_len + np.asarray(start_in_row, np.int64)[seg] + pos
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return flat, pos, cu


class PackedTokenizedCollator:
    """Pack examples into rows of max_length in arrival order, a new row whenever the
    next example does not fit; per-example causal boundaries are kept through
    cu_seqlens / unpad_indices / position_ids, and each segment's first token is
    excluded from the loss."""

    def __init__(self, max_length, pad_token_id):
        self.max_length = max_length
        self.pad_token_id = pad_token_id

    def __call__(self, examples):
        L = self.max_length
        seqs = [ex["token_ids"][:L] for ex in examples]
        seqs = [s for s in seqs if len(s)]
        lengths, row_of, start = [], [], []
        row, used = -1, 0
        for s in seqs:
            n = len(s)
            if row < 0 or used + n > L:
                row, used = row + 1, 0
            lengths.append(n)
            row_of.append(row)
            start.append(used)
            used += n
        B = row + 1
        flat, pos, cu = _segment_layout(lengths, row_of, start, L)
        input_ids = torch.full((B, L), self.pad_token_id, dtype=torch.long)
        attention_mask = torch.zeros((B, L), dtype=torch.bool)
        position_ids = torch.zeros((B, L), dtype=torch.long)
        if flat.size:
            fl = torch.from_numpy(flat)
            input_ids.view(-1)[fl] = torch.tensor([t for s in seqs for t in s], dtype=torch.long)
            attention_mask.view(-1)[fl] = True
            position_ids.view(-1)[fl] = torch.from_numpy(pos)
        loss_mask = attention_mask.clone()
        if lengths:
            heads = np.asarray(row_of, np.int64) * L + np.asarray(start, np.int64)
            loss_mask.view(-1)[torch.from_numpy(heads)] = False
        max_seqlen = max(lengths) if lengths else 0
        return {
            "input_ids": input_ids,
            "attention_mask": attention_mask,
            "loss_mask": loss_mask,
            "position_ids": position_ids,
            "cu_seqlens": torch.from_numpy(cu),
            "unpad_indices": torch.from_numpy(flat),
            "max_seqlen": min(((max_seqlen + 31) // 32) * 32, L),
        }


def sample_superposition_size(t: float, max_size: int) -> int:
    """Bag size s for training progress t in [0, 1]: max_size for t < 0.1, else 1
    (always 1 when max_size <= 1)."""
    if max_size <= 1:
        return 1
    return max_size if t < 0.1 else 1


def build_token_superposition_batch(batch, superposition_bag_size, latent_sequence_length, pad_token_id):
    """Fold each packed segment of a raw-token batch into bags of s tokens (bag j
    predicts the raw tokens of bag j + 1, never across a segment boundary), pack the
    bag segments into rows of latent_sequence_length by first-fit decreasing, and
    return the bag batch with MCCE labels [N, s] and s [N]; None when no segment has
    two full bags."""
    s_bag = int(superposition_bag_size)
    if s_bag <= 1:
        raise ValueError("superposition_bag_size must be > 1 for TST batches.")
    Ls = int(latent_sequence_length)
    input_ids = batch["input_ids"]
    cu = batch["cu_seqlens"].tolist()
    unpad = batch["unpad_indices"]
    flat_ids = input_ids.flatten()

    segs = []  # (source bags [n, s], n)
    for a, b in zip(cu[:-1], cu[1:]):
        full = (b - a) // s_bag
        if full < 2:
            continue
        bags = flat_ids[unpad[a:a + full * s_bag]].view(full, s_bag)[:Ls]
        if bags.size(0) - 1 == 0:
            continue
        segs.append(bags)
    if not segs:
        return None

    # first-fit decreasing; Python's sort is stable, so equal lengths keep arrival order
    order = sorted(range(len(segs)), key=lambda i: segs[i].size(0), reverse=True)
    row_fill, placed = [], []  # placed: (segment, row) in placement order
    for i in order:
        n = segs[i].size(0)
        for r, used in enumerate(row_fill):
            if used + n <= Ls:
                row_fill[r] += n
                placed.append((i, r))
                break
        else:
            row_fill.append(n)
            placed.append((i, len(row_fill) - 1))
    B = len(row_fill)
    # within a row, segments sit in placement order
    starts, cursor = [], [0] * B
    by_row = sorted(range(len(placed)), key=lambda j: placed[j][1])  # stable: placement order inside a row
    seg_seq = [placed[j] for j in by_row]
    for i, r in seg_seq:
        starts.append(cursor[r])
        cursor[r] += segs[i].size(0)
    lengths = [segs[i].size(0) for i, _ in seg_seq]
    rows = [r for _, r in seg_seq]
    flat, pos, cu_bags = _segment_layout(lengths, rows, starts, Ls)

    input_bags = torch.full((B, Ls, s_bag), pad_token_id, dtype=input_ids.dtype)
    attention_mask = torch.zeros((B, Ls), dtype=torch.bool)
    position_ids = torch.zeros((B, Ls), dtype=torch.long)
    fl = torch.from_numpy(flat)
    input_bags.view(B * Ls, s_bag)[fl] = torch.cat([segs[i] for i, _ in seg_seq], 0)
    attention_mask.view(-1)[fl] = True
    position_ids.view(-1)[fl] = torch.from_numpy(pos)
    labels = torch.cat([segs[i][1:] for i, _ in seg_seq], 0).contiguous()
    label_lengths = np.asarray(lengths, np.int64) - 1
    loss_flat, _, _ = _segment_layout(label_lengths, rows, starts, Ls)
    return {
        "input_ids": input_bags,
        "attention_mask": attention_mask,
        "position_ids": position_ids,
        "cu_seqlens": torch.from_numpy(cu_bags),
        "unpad_indices": torch.from_numpy(flat),
        "max_seqlen": bucket_max_seqlen(max(lengths), Ls),
        "loss_indices": torch.from_numpy(loss_flat),
        "labels": labels,
        "s": torch.full((labels.size(0),), s_bag, dtype=torch.int32),
    }


def bag_label_entropy_floor(labels, s):
    """Irreducible per-raw-token entropy of the target bags: per row, the entropy of the
    multiset of its first s labels, averaged with weights s."""
    if labels.numel() == 0:
        return torch.zeros((), device=labels.device, dtype=torch.float32)
    labels = labels.long()
    sf = s.float()
    active = torch.arange(labels.size(1), device=labels.device)[None, :] < s[:, None]
    srt = torch.where(active, labels, labels.new_full((), -1)).sort(dim=1).values
    live = srt >= 0
    new_run = live & torch.cat([torch.ones_like(srt[:, :1], dtype=torch.bool), srt[:, 1:] != srt[:, :-1]], dim=1)
    run = (new_run.cumsum(dim=1) - 1).clamp_min(0)
    counts = torch.zeros(labels.shape, dtype=torch.float32, device=labels.device)
    counts.scatter_add_(1, run, live.float())
    p = counts / sf[:, None].clamp_min(1.0)
    ent = torch.where(counts > 0, -p * torch.log(p.clamp_min(torch.finfo(torch.float32).tiny)), torch.zeros_like(p))
    return (ent.sum(-1) * sf).sum() / sf.sum().clamp_min(1.0)


def ce_equivalent_reducible_loss(raw_loss, vocab_size, entropy_floor):
    """Bag CE mapped onto the single-token CE scale: (loss - floor) * log V / (log V - floor);
    returns (rescaled loss, reducible gap)."""
    floor = entropy_floor.to(device=raw_loss.device, dtype=raw_loss.dtype).detach()
    random_loss = raw_loss.new_tensor(math.log(vocab_size))
    gap = (random_loss - floor).clamp_min(1e-6)
    return (raw_loss - floor) * (random_loss / gap), gap
