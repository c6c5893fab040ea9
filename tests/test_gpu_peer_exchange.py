"""The peer-memory exchange of the T-sharded stack.

* One GPU: all ranks' windows live in this process (PeerWindows.emulate) and
  the ranks' calls run one after another in stream order, so every wait is
  already satisfied when it runs.  The route must equal, bit for bit, the
  host route (stacked partial statistics + b200_gn_merge_ranks, halo frames
  copied by torch) and leave the fault word clear.
* One GPU: a wait nothing satisfies gives up after the wait limit, records
  its code in the fault word and (statistics) writes NaN -- the failure path
  a dead rank would take.
* 2+ GPUs (CUDA IPC across processes): exchange="peer" equals
  exchange="nccl" bit for bit, eagerly and through CUDA-graph replays.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from amd_tuned_torch import ops
from amd_tuned_torch import video_stack as vs
from amd_tuned_torch.peer import PeerWindows

pytestmark = pytest.mark.gpu


def _host_route(xs, sizes, params, i, backend):
    G = params.groups
    parts = torch.stack([backend.partial_stats(x, G) for x in xs])
    stats = ops.group_norm_merge_ranks(parts)
    xps = []
    for x in xs:
        N, C, T, H, W = x.shape
        xp = torch.zeros(N, T + 2, H, W, C, dtype=x.dtype, device=x.device)
        backend.norm_silu_into(x, stats, G, params.gn_weight[i], params.gn_bias[i], params.eps,
                               xp[:, 1:T + 1])
        xps.append(xp)
    R = len(xs)
    for r in range(R):
        if r > 0:
            xps[r][:, 0] = xps[r - 1][:, sizes[r - 1]]
        if r < R - 1:
            xps[r][:, sizes[r] + 1] = xps[r + 1][:, 1]
    return [backend.conv_cl(xp, params.conv_weight[i], params.conv_bias[i], 1) for xp in xps], stats


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("N,T,R", [(1, 7, 2), (2, 9, 3), (1, 12, 4), (1, 5, 4)])
def test_peer_route_emulated_matches_host_route(cuda, N, T, R, gated):
    C, H, W, G = 64, 8, 16, 8
    params = vs.make_params(channels=C, blocks=2, groups=G, dtype=torch.bfloat16, seed=3,
                            device=cuda)
    x = torch.randn(N, C, T, H, W, generator=torch.Generator().manual_seed(4))
    x = x.bfloat16().to(cuda)
    sizes = vs.t_partition(T, R)
    xs = list(torch.split(x, sizes, dim=2))
    xs = [t.contiguous() for t in xs]
    b = vs.CudaBackendInPlace()
    ops.read_device_flags(cuda)
    wins = PeerWindows.emulate(sizes, N * G, N, H, W, C, torch.bfloat16, cuda)
    try:
        yp, yh = xs, xs
        for i in range(2):
            for r in range(R):
                wins[r].publish(b.partial_stats(yp[r], G))
            stats = [wins[r].merge() for r in range(R)]
            for r in range(R):
                b.norm_silu_into(yp[r], stats[r], G, params.gn_weight[i], params.gn_bias[i],
                                 params.eps, wins[r].xp[:, 1:sizes[r] + 1])
            for r in range(R):
                wins[r].push()
            if not gated:
                for r in range(R):
                    wins[r].wait()
            yp = [b.conv_cl(wins[r].xp, params.conv_weight[i], params.conv_bias[i], 1,
                            gate=wins[r].gate() if gated else None)
                  for r in range(R)]
            yh, hstats = _host_route(yh, sizes, params, i, b)
            for r in range(R):
                assert torch.equal(stats[r], hstats), (i, r)
                assert torch.equal(yp[r], yh[r]), (i, r)
        torch.cuda.synchronize()
        assert ops.read_device_flags(cuda) == 0
    finally:
        for w in wins:
            w.close()


def test_peer_waits_time_out_into_fault_word(cuda):
    wins = PeerWindows.emulate([2, 2], 4, 1, 2, 8, 64, torch.bfloat16, cuda)
    try:
        ops.read_device_flags(cuda)
        wins[0].publish(torch.ones(4, 3, device=cuda))   # rank 1 never publishes
        out = wins[0].merge()
        torch.cuda.synchronize()
        assert torch.isnan(out).all()
        assert ops.read_device_flags(cuda) == 3
        wins[0].wait()                                   # rank 1 never pushes
        torch.cuda.synchronize()
        assert ops.read_device_flags(cuda) == 4
    finally:
        for w in wins:
            w.close()


def test_gated_conv_times_out_without_halo(cuda):
    """The conv's producer gives up on a halo that never arrives: fault code
    4, the kernel unwinds, and the context stays usable."""
    C, H, W, G = 64, 4, 16, 8
    params = vs.make_params(channels=C, blocks=1, groups=G, dtype=torch.bfloat16, seed=3,
                            device=cuda)
    wins = PeerWindows.emulate([3, 3], G, 1, H, W, C, torch.bfloat16, cuda)
    try:
        ops.read_device_flags(cuda)
        wins[0].publish(torch.ones(G, 3, device=cuda))   # epoch 1; rank 1 never pushes
        wins[0].xp.normal_()
        vs.CudaBackend().conv_cl(wins[0].xp, params.conv_weight[0], params.conv_bias[0], 1,
                                 gate=wins[0].gate())
        torch.cuda.synchronize()
        assert ops.read_device_flags(cuda) == 4
        # the context is still usable: an ungated conv runs and is finite
        y = vs.CudaBackend().conv_cl(wins[0].xp, params.conv_weight[0], params.conv_bias[0], 1)
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all()
        assert ops.read_device_flags(cuda) == 0
    finally:
        for w in wins:
            w.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_worker(rank, world, port, q):
    from datetime import timedelta
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        params = vs.make_params(channels=128, blocks=4, groups=32, dtype=torch.bfloat16,
                                seed=5, device=dev)
        x = torch.randn(1, 128, 13, 32, 32, generator=torch.Generator().manual_seed(9))
        xl = vs.shard_t(x.bfloat16(), rank, world).to(dev)
        y_nccl = vs.VideoStack(params, group=dist.group.WORLD).forward(xl)
        st = vs.VideoStack(params, group=dist.group.WORLD, exchange="peer")
        y_peer = st.forward(xl)
        st.capture(xl)
        g1 = st.replay().clone()
        g2 = st.replay().clone()
        torch.cuda.synchronize()
        res = {"eager": bool(torch.equal(y_peer, y_nccl)), "graph1": bool(torch.equal(g1, y_nccl)),
               "graph2": bool(torch.equal(g2, y_nccl)), "flags": ops.read_device_flags(dev)}
        st.close()
        out = [None] * world
        dist.all_gather_object(out, res)
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_equals_nccl_across_processes():
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=5)
    for r in res:
        assert r == {"eager": True, "graph1": True, "graph2": True, "flags": 0}, res
