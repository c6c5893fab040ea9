"""Video-VAE-decoder-like stack, optionally T-sharded across ranks.

    blocks x [GroupNorm(G) -> SiLU -> Conv3d(C, C, k=3, padding=1)]

on an [N, C, T, H, W] activation.  There is no reference counterpart: the
reference is single-GPU, and in a diffusion/VAE decoder these three ops are
separate F.group_norm / F.silu / F.conv3d calls, each through its own patched
tier.  This module runs the same math on this package's kernels and shards it
along T:

* GroupNorm statistics span all of T, so each rank computes partial
  (count, mean, M2) triples for its frames (b200_gn_partial_stats), the ranks
  all-gather them and every rank merges them in the same fixed order (Chan's
  pairwise update) -- identical statistics everywhere, independent of R.
* Normalise + SiLU is fused with the layout change the conv needs: it writes
  the channels-last conv operand straight into the interior frames of a
  buffer [N, T_local + 2, H, W, C] (b200_gn_apply).
* The two halo frames (k - 1 = 2 per layer: the neighbours' boundary frames)
  are exchanged between T-neighbours; the first and last rank zero theirs,
  which is exactly the conv's zero padding in T.
* Exchange routes: exchange="nccl" (all-gather + send/recv through
  torch.distributed) or exchange="peer" (peer.PeerWindows: the statistics
  and the halo frames are stored straight into the other GPUs' memory over
  NVLink and ordered by device flags -- no collective launch per block).
  Both give bit-identical results.
* conv3d on tensor cores (b200_conv3d_fwd, channels-last input) with T
  padding 0 over the haloed buffer produces the rank's T_local output frames.

`StackBackend` separates the host orchestration (partitioning, halo exchange,
statistics merge -- what the multi-process CPU tests check with gloo) from
the device kernels; `CudaBackend` is the only backend this package ships.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


@dataclass
class StackParams:
    gn_weight: List[torch.Tensor]
    gn_bias: List[torch.Tensor]
    conv_weight: List[torch.Tensor]
    conv_bias: List[torch.Tensor]
    groups: int = 32
    eps: float = 1e-5


def make_params(channels: int = 128, blocks: int = 4, groups: int = 32, eps: float = 1e-5,
                dtype: torch.dtype = torch.bfloat16, device="cpu", seed: int = 5) -> StackParams:
    """Random-init parameters: GroupNorm gamma = 1, beta = 0 (nn.GroupNorm's
    init); conv weight kaiming-uniform(a = sqrt(5)) and bias U(+-1/sqrt(fan_in))
    (nn.Conv3d's init), drawn from a seeded generator."""
    g = torch.Generator().manual_seed(seed)
    fan_in = channels * 27
    bound = 1.0 / math.sqrt(fan_in)
    gw, gb, cw, cb = [], [], [], []
    for _ in range(blocks):
        gw.append(torch.ones(channels, dtype=dtype, device=device))
        gb.append(torch.zeros(channels, dtype=dtype, device=device))
        w = (torch.rand(channels, channels, 3, 3, 3, generator=g) * 2 - 1) * bound
        b = (torch.rand(channels, generator=g) * 2 - 1) * bound
        cw.append(w.to(device=device, dtype=dtype))
        cb.append(b.to(device=device, dtype=dtype))
    return StackParams(gw, gb, cw, cb, groups, eps)


def t_partition(T: int, world: int) -> List[int]:
    """Frames per rank: as even as possible, earlier ranks take the remainder."""
    base, rem = divmod(T, world)
    return [base + (1 if r < rem else 0) for r in range(world)]


def merge_stats(parts: torch.Tensor) -> torch.Tensor:
    """Merge per-rank (count, mean, M2) triples [R, groups, 3] -> [groups, 3]
    in rank order (Chan et al.), fp64 internally."""
    parts = parts.double()
    n = parts[0, :, 0].clone()
    mean = parts[0, :, 1].clone()
    m2 = parts[0, :, 2].clone()
    for r in range(1, parts.shape[0]):
        nb, mb, qb = parts[r, :, 0], parts[r, :, 1], parts[r, :, 2]
        tot = n + nb
        safe = torch.where(tot > 0, tot, torch.ones_like(tot))
        d = mb - mean
        mean = torch.where(tot > 0, mean + d * nb / safe, mean)
        m2 = torch.where(tot > 0, m2 + qb + d * d * n * nb / safe, m2)
        n = tot
    return torch.stack([n, mean, m2], dim=1).float()


class StackBackend:
    """Device kernels the stack needs (one implementation per device kind)."""

    def partial_stats(self, x: torch.Tensor, groups: int) -> torch.Tensor:
        raise NotImplementedError

    def merge_ranks(self, parts: torch.Tensor) -> torch.Tensor:
        """[R, groups, 3] per-rank triples -> [groups, 3], rank order."""
        return merge_stats(parts).to(parts.device)

    def norm_silu_into(self, x: torch.Tensor, stats: torch.Tensor, groups: int,
                       weight, bias, eps: float, out_cl: torch.Tensor) -> None:
        """GroupNorm with `stats` + SiLU, written channels-last into out_cl
        ([N, T, H, W, C] contiguous view for one batch item at a time)."""
        raise NotImplementedError

    def conv_cl(self, xp: torch.Tensor, weight, bias, pad_hw: int, gate=None) -> torch.Tensor:
        """Conv3d over channels-last xp [N, Tp, H, W, C], T padding 0,
        H/W padding pad_hw; returns NCDHW [N, Cout, Tp - 2, H, W].  `gate`:
        halo arrival words the kernel waits on before the edge frames."""
        raise NotImplementedError


class CudaBackend(StackBackend):
    """This package's sm_100a kernels (libb200conv.so)."""

    def partial_stats(self, x, groups):
        from . import ops
        return ops.group_norm_partial_stats(x, groups)

    def merge_ranks(self, parts):
        from . import ops
        return ops.group_norm_merge_ranks(parts)

    def norm_silu_into(self, x, stats, groups, weight, bias, eps, out_cl):
        from . import ops
        N = x.shape[0]
        for n in range(N):
            y = ops.group_norm_apply(x[n:n + 1], stats[n * groups:(n + 1) * groups], groups,
                                     weight, bias, eps, silu=True, channels_last_out=True)
            out_cl[n].copy_(y.reshape(out_cl[n].shape))

    def conv_cl(self, xp, weight, bias, pad_hw, gate=None):
        from . import ops
        out = ops.conv3d(xp, weight, bias, (1, 1, 1), (0, pad_hw, pad_hw), (1, 1, 1),
                         x_channels_last=True, gate=gate)
        if out is None:
            raise RuntimeError("conv3d tensor-core kernel declined the stack's shape")
        return out


class CudaBackendInPlace(CudaBackend):
    """Like CudaBackend, but the normalise kernel writes directly into the
    interior of the haloed buffer (no staging copy) when the slice is
    contiguous."""

    def norm_silu_into(self, x, stats, groups, weight, bias, eps, out_cl):
        from . import _lib, ops
        L = _lib.lib()
        N, C = x.shape[0], x.shape[1]
        S = x[0].numel() // C
        for n in range(N):
            dst = out_cl[n]
            if not dst.is_contiguous():
                return super().norm_silu_into(x, stats, groups, weight, bias, eps, out_cl)
            adt = weight.dtype if weight is not None else x.dtype
            rc = L.b200_gn_apply(x[n].data_ptr(), stats[n * groups:].data_ptr(),
                                 ops._ptr(weight), ops._ptr(bias), dst.data_ptr(),
                                 ops._code(x.dtype), ops._code(adt), 1, C, S, groups,
                                 float(eps), 1, 1, ops._stream(x.device))
            if not _lib.check(rc, "b200_gn_apply"):
                raise _lib.NativeError("GroupNorm apply declined")


class VideoStack:
    """Runs the stack on one rank's T-slice (or the whole tensor when world == 1).

    `group` is a torch.distributed process group (None = no sharding).  All
    ranks call forward() with their own [N, C, T_local, H, W] slice; the
    result is the rank's slice of the output.
    """

    def __init__(self, params: StackParams, backend: Optional[StackBackend] = None,
                 group=None, exchange: str = "nccl"):
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', not {exchange!r}")
        self.p = params
        self.backend = backend or CudaBackendInPlace()
        self.group = group
        self.rank = dist.get_rank(group) if group is not None else 0
        self.world = dist.get_world_size(group) if group is not None else 1
        self.exchange = exchange
        self._peer = None

    # ------------------------------------------------------------ pieces
    def gn_stats(self, x: torch.Tensor) -> torch.Tensor:
        part = self.backend.partial_stats(x, self.p.groups).contiguous()   # [N*G, 3]
        if self.world == 1:
            return part
        # Concatenated along dim 0 (the form every backend accepts), then
        # viewed as [world, N*G, 3].
        gathered = torch.empty((self.world * part.shape[0],) + tuple(part.shape[1:]),
                               dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        return self.backend.merge_ranks(gathered.view((self.world,) + tuple(part.shape)))

    def exchange_halo(self, xp: torch.Tensor) -> None:
        """xp [N, T_local + 2, H, W, C]: send frame 1 to the previous rank and
        frame T_local to the next; receive into frames 0 and T_local + 1.
        The ends of the chain get zero frames (the conv's T padding)."""
        T = xp.shape[1] - 2
        prev_r = self.rank - 1 if self.rank > 0 else None
        next_r = self.rank + 1 if self.rank < self.world - 1 else None
        if prev_r is None:
            xp[:, 0].zero_()
        if next_r is None:
            xp[:, T + 1].zero_()
        if self.world == 1:
            return
        # For N == 1 a frame of xp is one contiguous block: send from and
        # receive into xp itself; otherwise through contiguous staging copies.
        direct = xp.shape[0] == 1 and xp.is_contiguous()
        ops_ = []
        staged = []
        def frame(t):
            return xp[:, t] if direct else xp[:, t].contiguous()
        if prev_r is not None:
            first = frame(1)
            ops_.append(dist.P2POp(dist.isend, first, self._global(prev_r), self.group))
            recv_lo = xp[:, 0] if direct else torch.empty_like(first)
            ops_.append(dist.P2POp(dist.irecv, recv_lo, self._global(prev_r), self.group))
            staged.append((0, recv_lo))
        if next_r is not None:
            last = frame(T)
            ops_.append(dist.P2POp(dist.isend, last, self._global(next_r), self.group))
            recv_hi = xp[:, T + 1] if direct else torch.empty_like(last)
            ops_.append(dist.P2POp(dist.irecv, recv_hi, self._global(next_r), self.group))
            staged.append((T + 1, recv_hi))
        for req in dist.batch_isend_irecv(ops_):
            req.wait()
        if not direct:
            for t, buf in staged:
                xp[:, t].copy_(buf)

    def _global(self, r: int) -> int:
        if self.group is None:
            return r
        return dist.get_global_rank(self.group, r)

    # -------------------------------------------------------- peer route
    def peer_windows(self, x: torch.Tensor):
        """The rank's peer window set, created (collectively) on first use for
        the activation shape of x."""
        if self._peer is None:
            from .peer import PeerWindows
            N, C, T, H, W = x.shape
            t_sizes: List[Optional[int]] = [None] * self.world
            dist.all_gather_object(t_sizes, int(T), group=self.group)
            self._peer = PeerWindows.create(self.group, N * self.p.groups, N, t_sizes, H, W, C,
                                            x.dtype, x.device)
        return self._peer

    def block_peer(self, x: torch.Tensor, i: int, pw=None) -> torch.Tensor:
        """One block over the peer windows `pw` (default: this rank's).  The
        halo push runs on a side stream while the conv computes its interior
        frames; the conv's producer waits for the halo arrivals itself
        before the edge frames (b200_conv3d_fwd_gated)."""
        T = x.shape[2]
        pw = pw or self.peer_windows(x)
        pw.publish(self.backend.partial_stats(x, self.p.groups))
        stats = pw.merge()
        self.backend.norm_silu_into(x, stats, self.p.groups, self.p.gn_weight[i],
                                    self.p.gn_bias[i], self.p.eps, pw.xp[:, 1:T + 1])
        main = torch.cuda.current_stream(x.device)
        side = self._side_stream(x.device)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            pw.push()
        y = self.backend.conv_cl(pw.xp, self.p.conv_weight[i], self.p.conv_bias[i], 1,
                                 gate=pw.gate())
        main.wait_stream(side)      # the next block's apply overwrites what the push reads
        return y

    def _side_stream(self, device) -> torch.cuda.Stream:
        s = getattr(self, "_side", None)
        if s is None:
            s = self._side = torch.cuda.Stream(device=device)
        return s

    # -------------------------------------------------------------- main
    def block(self, x: torch.Tensor, i: int) -> torch.Tensor:
        if self.exchange == "peer" and self.world > 1:
            return self.block_peer(x, i)
        N, C, T, H, W = x.shape
        stats = self.gn_stats(x)
        xp = torch.empty(N, T + 2, H, W, C, dtype=x.dtype, device=x.device)
        self.backend.norm_silu_into(x, stats, self.p.groups, self.p.gn_weight[i],
                                    self.p.gn_bias[i], self.p.eps, xp[:, 1:T + 1])
        self.exchange_halo(xp)
        return self.backend.conv_cl(xp, self.p.conv_weight[i], self.p.conv_bias[i], 1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        for i in range(len(self.p.conv_weight)):
            x = self.block(x, i)
        return x

    # --------------------------------------------------------- CUDA graph
    def capture(self, x: torch.Tensor) -> torch.Tensor:
        """Captures one forward step on the static input `x` (kernels and the
        NCCL statistics gather / halo send-recv) into a CUDA graph; returns
        the graph's output tensor.  replay() re-runs the step with no host
        launch work -- the sharded stack is otherwise bound by the host
        issuing ~10 launches and collectives per block.  Every rank must
        capture (the collectives inside pair up across ranks); call release()
        before the process group is destroyed."""
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                self.forward(x)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        if self.group is not None:
            dist.barrier(group=self.group)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self._graph_out = self.forward(x)
        torch.cuda.synchronize(x.device)
        return self._graph_out

    def replay(self) -> torch.Tensor:
        self._graph.replay()
        return self._graph_out

    def release(self) -> None:
        self._graph = None
        self._graph_out = None

    def close(self) -> None:
        """Drops the graph and, collectively, the peer windows; call before
        the process group is destroyed."""
        self.release()
        if self._peer is not None:
            self._peer.close(self.group)
            self._peer = None


def reference_forward(x: torch.Tensor, params: StackParams,
                      round_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """The stack in plain torch ops (F.group_norm / F.silu / F.conv3d), fp32
    math; with round_dtype, activations are rounded to it at the same op
    boundaries as the device path (after GN+SiLU and after each conv)."""
    import torch.nn.functional as F
    h = x.float()
    for i in range(len(params.conv_weight)):
        h = F.group_norm(h, params.groups, params.gn_weight[i].float(),
                         params.gn_bias[i].float(), params.eps)
        h = F.silu(h)
        if round_dtype is not None:
            h = h.to(round_dtype).float()
        h = F.conv3d(h, params.conv_weight[i].float(), params.conv_bias[i].float(), padding=1)
        if round_dtype is not None:
            h = h.to(round_dtype).float()
    return h


def shard_t(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's T-slice of [N, C, T, H, W]."""
    sizes = t_partition(x.shape[2], world)
    start = sum(sizes[:rank])
    return x[:, :, start:start + sizes[rank]].contiguous()


def shard_dim(x: torch.Tensor, dim: int, rank: int, world: int) -> torch.Tensor:
    """Batch/channel sharding with no communication (the other BASELINE
    configs): this rank's contiguous slice along `dim`."""
    sizes = t_partition(x.shape[dim], world)
    start = sum(sizes[:rank])
    return x.narrow(dim, start, sizes[rank])
