"""Fleet mode: many independent robot requests sharded over the GPUs of a box.

Each request is one batch-1 sampler call with its own prefix and noise
(``ActionExpert.sample(prefix, steps, x0)``); requests never exchange data, so
the fleet is split into contiguous blocks of requests, one block per rank (one
process per GPU), with no collective on the data path. Inside a rank the block
runs as sampler calls over chunks of ``chunk`` requests (every GEMM of a call
sees 50 * chunk tokens): small chunks as the single fused launch, large ones
layer by layer on the tcgen05 dequant-GEMM (``flow_sample`` picks). On a CUDA
device each chunk's whole 10-step call is captured once as a CUDA graph
(``GraphedSampler`` with the chunk's own prefix K/V), so a fleet step replays
one graph per chunk instead of dispatching every kernel of the layer-by-layer
path from Python.
Results come back through host memory; ``gather_results`` assembles the whole
fleet on one rank over any process group (gloo included) when a caller wants
it, and is not part of the timed path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch


def shard_bounds(n_requests: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of request indices owned by `rank` (the first
    n_requests % world ranks get one extra request)."""
    if world < 1 or not (0 <= rank < world) or n_requests < 0:
        raise ValueError(f"bad shard request: n={n_requests} rank={rank} world={world}")
    base, extra = divmod(n_requests, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def chunk_bounds(lo: int, hi: int, chunk: int) -> list[tuple[int, int]]:
    """[lo, hi) cut into consecutive pieces of at most `chunk` requests."""
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    return [(a, min(a + chunk, hi)) for a in range(lo, hi, chunk)]


@dataclass
class FleetShard:
    lo: int
    hi: int
    actions: torch.Tensor  # [hi - lo, horizon, action_dim], on the host


class FleetSampler:
    """Runs this rank's block of a fleet of ``n_requests`` sampler requests.

    ``request_fn(i)`` returns request i's (prefix [1, P, d], noise [1, H, A])
    (the caller decides where requests come from; ``synth.fleet_request``
    gives the seeded synthetic fleet). With an
    ``expert`` the chunks run through ``flow_sample`` (one fused launch per
    chunk); ``sample_fn(prefix[B,P,d], x0[B,H,A]) -> actions[B,H,A]`` replaces
    it (the host logic is then testable without a GPU).
    """

    def __init__(self, n_requests: int, rank: int, world: int, chunk: int = 256, n_steps: int = 10,
                 expert=None, sample_fn: Optional[Callable] = None, device=None, graphs: bool = True):
        if (expert is None) == (sample_fn is None):
            raise ValueError("give exactly one of expert / sample_fn")
        self.n, self.rank, self.world = n_requests, rank, world
        self.chunk, self.n_steps = chunk, n_steps
        self.lo, self.hi = shard_bounds(n_requests, rank, world)
        self.expert, self.sample_fn = expert, sample_fn
        self.device = device
        self.graphs = graphs
        self._inputs = None
        self._graphs = None

    def stage(self, request_fn: Callable[[int], tuple]):
        """Build this rank's chunks once: per chunk the stacked prefixes and
        noise on the device and, with an expert, the encoded prefix K/V."""
        staged = []
        for a, b in chunk_bounds(self.lo, self.hi, self.chunk):
            reqs = [request_fn(i) for i in range(a, b)]
            pre = torch.cat([r[0] for r in reqs], 0)
            x0 = torch.cat([r[1] for r in reqs], 0)
            if self.device is not None:
                pre, x0 = pre.to(self.device), x0.to(self.device)
            kv = None
            if self.expert is not None:
                dt = self.expert.out_norm.weight.dtype
                pre, x0 = pre.to(dt), x0.to(dt)
                kv = self.expert.encode(pre)
            staged.append((a, b, pre, x0, kv))
        self._inputs = staged
        self._graphs = None
        if self.expert is not None and self.graphs and staged and staged[0][3].is_cuda:
            from .graphed import GraphedSampler
            self._graphs = [GraphedSampler(self.expert, x0, self.n_steps, warmup=2, prefix_kv=kv)
                            for _, _, _, x0, kv in staged]
        return self

    def run_device(self) -> list[torch.Tensor]:
        """One fleet step on this rank: every chunk's sampler call, results
        left on the device (no host synchronisation)."""
        if self._inputs is None:
            raise RuntimeError("stage() the requests first")
        if self._graphs is not None:
            # one replay per chunk; each output is the chunk graph's static
            # buffer, overwritten by its next replay
            return [g.replay() for g in self._graphs]
        outs = []
        for a, b, pre, x0, kv in self._inputs:
            if self.expert is not None:
                from .expert import flow_sample
                outs.append(flow_sample(self.expert, x0, self.n_steps, kv))
            else:
                outs.append(self.sample_fn(pre, x0))
        return outs

    def run(self) -> FleetShard:
        """One fleet step, results copied to the host."""
        outs = self.run_device()
        acts = torch.cat([o.float().cpu() for o in outs], 0) if outs else torch.empty(0)
        return FleetShard(self.lo, self.hi, acts)


def gather_results(shard: FleetShard, n_requests: int, group=None, dst: int = 0) -> Optional[torch.Tensor]:
    """Assemble every rank's shard on rank `dst` over a process group (any
    backend); returns the [n_requests, H, A] actions there and None elsewhere.
    Result collection only -- the sampler path itself has no collective."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return shard.actions
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    objs: Sequence = [None] * world if rank == dst else None
    dist.gather_object((shard.lo, shard.hi, shard.actions), objs, dst=dst, group=group)
    if rank != dst:
        return None
    parts = sorted(objs, key=lambda o: o[0])
    out = torch.cat([p[2] for p in parts if p[1] > p[0]], 0)
    if out.shape[0] != n_requests:
        raise RuntimeError(f"fleet gather got {out.shape[0]} of {n_requests} requests")
    return out
