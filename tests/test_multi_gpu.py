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
* ExpertParallelGLUMLP on one rank (no exchange) against GLUMLP;
* CopyEngineAllReduce (copy-engine all-reduce over CUDA IPC peer memory):
  bit-exact against the f32 sum in rank order, rounded once, over several
  steps, bf16 and f32, sizes that do not split evenly; GradAllReducer with
  engine="ce" against engine="nccl" on a small model; and a peer that never
  joins: the bounded wait expires and records ZS_DEVERR_TIMEOUT_PEER instead
  of hanging.
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


def _ce_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from zs_b200.ce import CopyEngineAllReduce
        from zs_b200 import device_error

        dev = torch.device("cuda", rank)
        ok = []
        for dt, n in ((torch.bfloat16, 1_000_003), (torch.float32, 77_777), (torch.bfloat16, 9)):
            ce = CopyEngineAllReduce(n, dt)
            for step in range(3):
                g = torch.Generator(device=dev).manual_seed(100 * step + n)
                xs = [torch.randn(n, device=dev, generator=g).to(dt) for _ in range(world)]
                scale = 0.5 if step == 1 else 1.0
                acc = xs[0].float()
                for r in range(1, world):
                    acc = acc + xs[r].float()
                want = (acc * scale).to(dt)
                t = xs[rank].clone()
                ce(t, scale=scale)
                torch.cuda.synchronize()
                ok.append(bool(torch.equal(t, want)))
            ce.close()
        err = device_error()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, err, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def _reducer_ce_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from zs_b200.dp import GradAllReducer

        dev = torch.device("cuda", rank)
        torch.manual_seed(0)
        nets = [torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.GELU(), torch.nn.Linear(128, 32)).to(dev)
                for _ in range(2)]
        nets[1].load_state_dict(nets[0].state_dict())
        reds = [GradAllReducer(list(nets[0].parameters()), bucket_mb=0.01, average=True, engine="nccl"),
                GradAllReducer(list(nets[1].parameters()), bucket_mb=0.01, average=True, engine="ce")]
        worst = 0.0
        same_ranks = True
        for step in range(3):
            g = torch.Generator(device=dev).manual_seed(10 * step + rank)
            x = torch.randn(16, 64, device=dev, generator=g)
            for net, red in zip(nets, reds):
                net.zero_grad(set_to_none=True)
                net(x).square().sum().backward()
                red.finish()
            for a, b in zip(nets[0].parameters(), nets[1].parameters()):
                worst = max(worst, _rel(b.grad, a.grad))
            flat = torch.cat([p.grad.flatten() for p in nets[1].parameters()])
            allf = [torch.empty_like(flat) for _ in range(world)]
            dist.all_gather(allf, flat)
            same_ranks = same_ranks and all(torch.equal(f, allf[0]) for f in allf)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, worst, same_ranks, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def _ce_timeout_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from zs_b200.ce import CopyEngineAllReduce
        from zs_b200 import _lib as Z
        from zs_b200 import device_error

        ce = CopyEngineAllReduce(4096, torch.float32)
        err = 0
        if rank == 0:
            # rank 1 never calls: the waits for its flags run out (about a second each)
            t = torch.ones(4096, device=torch.device("cuda", rank))
            ce(t)
            torch.cuda.synchronize()
            err = device_error()
            Z.clear_device_error()
        dist.barrier()
        ce.close()
        dist.destroy_process_group()
        q.put((rank, err, None, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def test_ce_allreduce_two_gpus_bit_exact():
    for rank, ok, err, tb in _spawn(_ce_worker):
        assert tb is None, tb
        assert err == 0
        assert all(ok), f"rank {rank}: {ok}"


def test_grad_reducer_copy_engine_two_gpus():
    for rank, worst, same_ranks, tb in _spawn(_reducer_ce_worker):
        assert tb is None, tb
        assert same_ranks, f"rank {rank}: reduced gradients differ across ranks"
        assert worst < 1e-5, f"rank {rank}: copy-engine vs NCCL gradients differ by {worst:.3e}"


def test_ce_allreduce_peer_timeout_is_reported():
    for rank, err, _, tb in _spawn(_ce_timeout_worker):
        assert tb is None, tb
        if rank == 0:
            assert err & 0x20, f"expected ZS_DEVERR_TIMEOUT_PEER, got {err:#x}"


def _ep1_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from scattermoe.expert_parallel import ExpertParallelGLUMLP
        from scattermoe.mlp import GLUMLP

        dev = torch.device("cuda", rank)
        T, d, E, k, f = 700, 128, 8, 3, 64
        g = torch.Generator(device=dev).manual_seed(8)
        x = torch.randn(T, d, device=dev, generator=g).bfloat16()
        p, idx = torch.sigmoid(torch.randn(T, E, device=dev, generator=g)).topk(k, dim=-1)
        p = p.bfloat16()
        dy = torch.randn(T, d, device=dev, generator=g).bfloat16()
        full = GLUMLP(d, f, E, k).to(dev).bfloat16()
        ep = ExpertParallelGLUMLP(d, f, E, k).to(dev).bfloat16().load_from_full(full)
        outs = []
        for m in (full, ep):
            xr, pr = x.clone().requires_grad_(True), p.clone().requires_grad_(True)
            y = m(xr, pr, idx)
            y.backward(dy)
            outs.append((y, xr.grad, pr.grad, m.experts.weight.grad, m.output_experts.weight.grad))
        res = [(_rel(a, b), _cos(a, b)) for a, b in zip(outs[1], outs[0])]
        dist.destroy_process_group()
        q.put((rank, res, None, None))
    except Exception:
        import traceback

        q.put((rank, None, None, traceback.format_exc()))


def test_expert_parallel_single_rank_equals_glumlp():
    for rank, res, _, tb in _spawn(_ep1_worker, world=1):
        assert tb is None, tb
        for rel, cos in res:
            assert rel < 1e-2 and cos > 0.999, res
