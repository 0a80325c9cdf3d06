"""Two-GPU paths over NCCL (skipped with fewer than two GPUs):

* ExpertParallelGLUMLP (experts split over two ranks, dispatch/combine
  all-to-all) against one GPU running GLUMLP with all experts on both ranks'
  tokens: outputs, token and routing-weight gradients, expert weight gradients;
  bf16 tolerance (relative L2 error <= 1e-2, cosine >= 0.999);
* MuonMDWithAuxAdam (Newton-Schulz split over the ranks, all-gathered) against
  SingleDeviceMuonMDWithAuxAdam: parameters bit-identical on both ranks after
  two steps, and within 1e-5 relative of the single-device optimizer (a rank's
  Newton-Schulz batch holds fewer matrices, which can change the kernels' tile
  split and so the f32 accumulation order of the bf16 GEMMs).
Ranks are child processes, one per GPU, with a short process-group timeout."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _cos(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _init(rank, world, port):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))


def _ep_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from scattermoe.expert_parallel import ExpertParallelGLUMLP
        from scattermoe.mlp import GLUMLP
        from zs_b200 import device_error

        dev = torch.device("cuda", rank)
        T, d, E, k, f = 512, 256, 16, 4, 128
        g = torch.Generator(device=dev).manual_seed(5)
        bf = torch.bfloat16
        x = torch.randn(world, T, d, device=dev, generator=g).to(bf)
        logits = torch.randn(world, T, E, device=dev, generator=g)
        logits[..., :4] += 1.5  # skewed loads
        p, idx = torch.sigmoid(logits).topk(k, dim=-1)
        p = (p / p.sum(-1, keepdim=True)).to(bf)
        dy = torch.randn(world, T, d, device=dev, generator=g).to(bf)
        full = GLUMLP(d, f, E, k).to(dev)
        with torch.no_grad():
            full.experts.weight.normal_(0, 0.05, generator=g)
            full.output_experts.weight.normal_(0, 0.05, generator=g)
        full = full.to(bf)
        xf = x.reshape(world * T, d).clone().requires_grad_(True)
        pf = p.reshape(world * T, k).clone().requires_grad_(True)
        yf = full(xf, pf, idx.reshape(world * T, k))
        yf.backward(dy.reshape(world * T, d))

        ep = ExpertParallelGLUMLP(d, f, E, k).to(dev).to(bf).load_from_full(full)
        xr = x[rank].clone().requires_grad_(True)
        pr = p[rank].clone().requires_grad_(True)
        y = ep(xr, pr, idx[rank])
        y.backward(dy[rank])
        torch.cuda.synchronize()
        sl = slice(rank * T, (rank + 1) * T)
        el = E // world
        es = slice(rank * el, (rank + 1) * el)
        pairs = {"y": (y, yf[sl]), "dx": (xr.grad, xf.grad[sl]), "dp": (pr.grad, pf.grad[sl]),
                 "dW1": (ep.experts.weight.grad, full.experts.weight.grad[es]),
                 "dW2": (ep.output_experts.weight.grad, full.output_experts.weight.grad[es])}
        res = {n: (_rel(a, b), _cos(a, b)) for n, (a, b) in pairs.items()}
        err = device_error()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res, err, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def _muon_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from optimizer.muon import MuonMDWithAuxAdam, SingleDeviceMuonMDWithAuxAdam

        dev = torch.device("cuda", rank)
        shapes = [(256, 512), (512, 256), (6, 384, 256), (3, 256, 256), (1, 128, 640), (64,)]

        def make():
            g = torch.Generator(device=dev).manual_seed(9)
            ps = [torch.nn.Parameter(torch.randn(s, device=dev, generator=g) * 0.02) for s in shapes]
            grads = [[torch.randn(s, device=dev, generator=g) for s in shapes] for _ in range(2)]
            return ps, grads

        def run(cls, *extra):
            ps, grads = make()
            t = lambda v: torch.tensor(v, device=dev)  # noqa: E731
            opt = cls([dict(params=ps[:5], use_muon=True, lr=t(0.02), capturable=True),
                       dict(params=ps[5:], use_muon=False, lr=t(3e-4), capturable=True)], *extra)
            for gs in grads:
                for p_, g_ in zip(ps, gs):
                    p_.grad = g_.clone()
                opt.step()
            torch.cuda.synchronize()
            return [p_.detach().clone() for p_ in ps]

        ref = run(SingleDeviceMuonMDWithAuxAdam)
        got = run(MuonMDWithAuxAdam, dist.group.WORLD)
        worst = max(_rel(a, b) for a, b in zip(got, ref))
        # the replicas stay in sync: every rank holds the same bits
        mine = torch.cat([p_.flatten() for p_ in got])
        others = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(others, mine)
        same = all(torch.equal(o, others[0]) for o in others)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, same, worst, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def _spawn(worker, world=2):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return res


def test_expert_parallel_glumlp_two_gpus():
    for rank, res, err, tb in _spawn(_ep_worker):
        assert tb is None, tb
        assert err == 0
        for name, (rel, cos) in res.items():
            assert rel < 1e-2 and cos > 0.999, f"rank {rank} {name}: rel {rel:.3e} cos {cos:.6f}"


def test_sharded_muonmd_two_gpus():
    for rank, same, worst, tb in _spawn(_muon_worker):
        assert tb is None, tb
        assert same, f"rank {rank}: the ranks' parameters differ"
        assert worst < 1e-5, f"rank {rank}: worst relative error {worst:.3e} against the single-device optimizer"
