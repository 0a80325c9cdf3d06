"""Expert-parallel GLUMLP host logic on CPU with gloo ranks: the global sort, the
count exchange, the dispatch/combine all-to-alls and their autograd adjoints.
The device functions (gather, slot sum, GLU experts, sort) are replaced by
plain-torch restatements of the same math so the test runs without a GPU; the
result on every rank must equal one process running all experts on the
concatenation of all ranks' tokens (GLUMLP semantics, scattermoe/mlp.py:74-95):
outputs, token and routing-weight gradients on the token's rank, expert weight
gradients on the expert's rank.  Cases: skewed routing, a rank whose experts
receive no rows, and world sizes 2 and 4."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _t_sort(idx, E):
    flat = idx.reshape(-1)
    sei, ssi = torch.sort(flat, stable=True)
    offs = torch.cumsum(torch.bincount(flat, minlength=E), 0)
    return sei, ssi, offs


def _t_gather(x, ssi, k):
    return x[ssi // k]


def _t_slot_sum(rows, ssi, T, k):
    slot = torch.zeros((T * k,) + tuple(rows.shape[1:]), dtype=rows.dtype).index_copy(0, ssi, rows)
    return slot.view(T, k, -1).sum(1)


def _t_experts(x, p, lid, W1, W2, E, fuse):
    """GLU experts with k = 1: y = p * (silu(x W1[e]_gate) * x W1[e]_up) W2[e]^T."""
    lid = lid.reshape(-1)
    f = W2.size(2)
    h = torch.einsum("rd,rod->ro", x, W1[lid])
    a = torch.nn.functional.silu(h[:, f:]) * h[:, :f]
    y = torch.einsum("rf,rdf->rd", a, W2[lid])
    return y * p.reshape(-1, 1)


KERNELS = dict(gather=_t_gather, slot_sum=_t_slot_sum, experts=_t_experts, sort=_t_sort)


def _inputs(world, T, d, E, k, f, empty_rank):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(world, T, d, generator=g, dtype=torch.float64)
    logits = torch.randn(world, T, E, generator=g, dtype=torch.float64)
    logits[..., : E // 4] += 2.0  # skewed loads
    if empty_rank is not None:
        el = E // world
        logits[..., empty_rank * el:(empty_rank + 1) * el] = -1e9
    p, idx = torch.sigmoid(logits).topk(k, dim=-1)
    p = p / p.sum(-1, keepdim=True)
    W1 = torch.randn(E, 2 * f, d, generator=g, dtype=torch.float64) * 0.2
    W2 = torch.randn(E, d, f, generator=g, dtype=torch.float64) * 0.2
    dy = torch.randn(world, T, d, generator=g, dtype=torch.float64)
    return x, p, idx, W1, W2, dy


def _full(x, p, idx, W1, W2, dy, E, k):
    """One process, all experts, all tokens: GLUMLP forward and backward."""
    x = x.reshape(-1, x.size(-1)).clone().requires_grad_(True)
    p = p.reshape(-1, k).clone().requires_grad_(True)
    W1 = W1.clone().requires_grad_(True)
    W2 = W2.clone().requires_grad_(True)
    T = x.size(0)
    _, ssi, _ = _t_sort(idx.reshape(-1, k), E)
    rows = _t_experts(_t_gather(x, ssi, k), p.reshape(-1)[ssi], idx.reshape(-1)[ssi], W1, W2, E, False)
    y = _t_slot_sum(rows, ssi, T, k)
    y.backward(dy.reshape(T, -1))
    return y.detach(), x.grad, p.grad, W1.grad, W2.grad


def _worker(rank, world, port, empty_rank, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        from scattermoe.expert_parallel import ExpertParallelGLUMLP

        T, d, E, k, f = 24, 8, 8, 3, 6
        x, p, idx, W1, W2, dy = _inputs(world, T, d, E, k, f, empty_rank)
        ry, rdx, rdp, rdW1, rdW2 = _full(x, p, idx, W1, W2, dy, E, k)

        layer = ExpertParallelGLUMLP(d, f, E, k, kernels=KERNELS).double()
        el = E // world
        with torch.no_grad():
            layer.experts.weight.copy_(W1[rank * el:(rank + 1) * el])
            layer.output_experts.weight.copy_(W2[rank * el:(rank + 1) * el])
        xr = x[rank].clone().requires_grad_(True)
        pr = p[rank].clone().requires_grad_(True)
        y = layer(xr, pr, idx[rank])
        y.backward(dy[rank])
        sl = slice(rank * T, (rank + 1) * T)
        errs = {
            "y": (y.detach() - ry[sl]).abs().max().item(),
            "dx": (xr.grad - rdx[sl]).abs().max().item(),
            "dp": (pr.grad - rdp[sl]).abs().max().item(),
            "dW1": (layer.experts.weight.grad - rdW1[rank * el:(rank + 1) * el]).abs().max().item(),
            "dW2": (layer.output_experts.weight.grad - rdW2[rank * el:(rank + 1) * el]).abs().max().item(),
        }
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("world,empty_rank", [(2, None), (2, 1), (4, None), (4, 2)])
def test_expert_parallel_glumlp_matches_single_process(world, empty_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, empty_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, err in res:
        assert err is None, err
        for name, e in errs.items():
            assert e < 1e-12, f"rank {rank}: {name} differs by {e}"


def _shard_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        from zs_b200.lm import MoELM as MoEModel
        from modeling.model_config import ModelConfig
        from scattermoe.expert_parallel import ExpertParallelGLUMLP, shard_experts

        cfg = ModelConfig(vocab_size=64, embed_size=32, hidden_size=32, transformer_depth=2, intermediate_size=16,
                          n_experts=9, n_shared_experts=1, n_experts_per_token=2, n_attention_heads=2,
                          n_key_value_heads=1, attention_window_pattern=(None, None), max_position_embeddings=32,
                          sequence_length=32, pos_rope_dims=8)
        torch.manual_seed(0)
        model = MoEModel(cfg)
        full = {n: p.detach().clone() for n, p in model.named_parameters()}
        eps = shard_experts(model)
        ok = len(eps) == 2 and all(isinstance(l.mlp.routed_experts, ExpertParallelGLUMLP) for l in model.layers)
        el = 8 // world
        for n, p in model.named_parameters():
            if "routed_experts" in n:
                ok = ok and torch.equal(p, full[n][rank * el:(rank + 1) * el])
            else:
                ok = ok and torch.equal(p, full[n])
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception:  # pragma: no cover
        import traceback

        q.put((rank, False, traceback.format_exc()))


def test_shard_experts_module_surgery():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert err is None, err
        assert ok, f"rank {rank}: sharded parameters differ from the full model's slice"
