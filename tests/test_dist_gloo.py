"""Multi-rank host logic of the sharded Muon step over ``gloo`` on CPU.

Two ranks build the same ``ShardLayout``; each applies a stand-in update
(the GPU kernels need a device) to its own slot only, then ``exchange()``
all-gathers in place. Every rank must end with every matrix updated once.
A rank that leaves before the collective is reported to the other through
the process-group timeout instead of hanging it.
"""

import datetime
import os
import socket
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHAPES = [(64, 96), (96, 64), (64, 96), (32, 32), (64, 96), (16, 48), (128, 16)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_exchange(rank, world, port, q):
    try:
        from pytorch_opt_b200.dist import ShardLayout, ShardedMuon
        _init(rank, world, port)
        lay = ShardLayout(SHAPES, world)
        params = torch.zeros(lay.numel)
        grads = torch.zeros(lay.numel)
        for i in range(len(SHAPES)):
            lay.matrix(grads, i).fill_(float(i + 1))
        touched = []

        def fake_update(p, g):  # stands in for the grouped Muon kernels
            p.add_(g)
            touched.append(p.shape[0])

        sm = ShardedMuon(lay, params, grads, rank, compute=fake_update)
        sm.step()
        ok = all(torch.all(lay.matrix(params, i) == float(i + 1)) for i in range(len(SHAPES)))
        n_local = sum(touched)
        # The host-gradient step: the same update again from a slot-shaped copy.
        host = lay.slot_tensor(grads, rank)
        grads.zero_()
        sm.step_from_host(host)
        ok = ok and all(torch.all(lay.matrix(params, i) == 2.0 * (i + 1)) for i in range(len(SHAPES)))
        q.put((rank, bool(ok), n_local, len(lay.assign[rank])))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, traceback.format_exc(), -1))


def _worker_band_syrk(rank, world, port, q):
    try:
        from pytorch_opt_b200.dist import sharded_syrk_ema_
        _init(rank, world, port)
        g = torch.Generator().manual_seed(5)
        X = torch.randn(64, 300, generator=g, dtype=torch.float64)
        F = torch.zeros(300, 300, dtype=torch.float64)

        def band_matmul(band, X, r0, r1, a, b):  # stands in for the tensor-core band product
            band.mul_(b).add_(a * (X[:, r0:r1].T @ X[:, :r1]))

        F32 = F.float()
        sharded_syrk_ema_(F32, X.float(), 0.5, 0.9, True, rank, world, compute=band_matmul)
        ok1 = torch.allclose(F32.double(), 0.5 * X.T @ X, rtol=1e-5, atol=1e-5)
        X2 = torch.randn(64, 300, generator=g, dtype=torch.float64)
        want = 0.9 * F32.double() + 0.1 * 0.5 * X2.T @ X2
        sharded_syrk_ema_(F32, X2.float(), 0.5, 0.9, False, rank, world, compute=band_matmul)
        ok2 = torch.allclose(F32.double(), want, rtol=1e-5, atol=1e-5) and torch.equal(F32, F32.T)
        q.put((rank, bool(ok1 and ok2)))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_factor_sharding(rank, world, port, q):
    try:
        from pytorch_opt_b200.dist import sharded_factor_updates_
        _init(rank, world, port)
        g = torch.Generator().manual_seed(6)
        Xs = [torch.randn(32, d, generator=g, dtype=torch.float64) for d in (20, 12, 30)]
        Fs = [torch.full((X.shape[1], X.shape[1]), float("nan"), dtype=torch.float64) for X in Xs]

        def syrk_ema(F, X, alpha, beta, first):  # stands in for the fused kernel
            S = alpha * X.T @ X
            F.copy_(S if first else beta * F + (1 - beta) * S)

        owners = sharded_factor_updates_([(F, X, 0.5, 0.9, True) for F, X in zip(Fs, Xs)], rank, world,
                                         compute=syrk_ema)
        ok = sorted(set(owners)) == list(range(world))
        ok = ok and all(torch.allclose(F, 0.5 * X.T @ X) for F, X in zip(Fs, Xs))  # every factor on every rank
        q.put((rank, bool(ok)))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_dead_peer(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before leaving abruptly
            os._exit(0)  # leaves between steps, without joining the collective
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            q.put((rank, "no-error"))
        except Exception as e:  # the survivor learns of it on the host
            q.put((rank, "error:" + type(e).__name__))
    except Exception:
        q.put((rank, "setup-failed:" + traceback.format_exc()))


def _run(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_sharded_exchange_two_ranks():
    res = _run(_worker_exchange, 2)
    for rank, ok, n_local, n_assigned in res:
        assert ok is True, n_local
        assert n_local == n_assigned  # each rank updated exactly its own matrices
    assert res[0][3] + res[1][3] == len(SHAPES)


def test_dead_peer_surfaces_as_host_error():
    res = _run(_worker_dead_peer, 2)
    assert res[1][1] == "left"
    assert res[0][1].startswith("error:"), res[0][1]


def test_band_split_factor_update_two_ranks():
    res = _run(_worker_band_syrk, 2)
    assert res[0][1] is True and res[1][1] is True, res



def test_factor_sharding_two_ranks():
    """Whole factors per rank (LPT), each broadcast from its owner: every rank
    ends with every updated factor, and both ranks own work."""
    res = _run(_worker_factor_sharding, 2)
    assert res[0][1] is True and res[1][1] is True, res
