"""Expert parallelism for the MoE layer across the GPUs of one node.

The reference runs the whole layer on one device (its MoE call is
CudaDevice::moe_topk_batch_q4_0, crates/mrml-tensor/src/cuda.rs:2840-2880,
and nothing in it communicates).  Here the experts are sharded: rank r of P
holds the contiguous experts [r*E/P, (r+1)*E/P) and owns T "home" tokens.
One layer step on every rank:

1. route the home tokens with the replicated router (mrml_moe_router);
2. dispatch: all-gather the home tokens' rows, expert ids and weights, so
   every rank sees all P*T tokens;
3. compute: mrml_moe_experts_shard over the P*T tokens, which skips the
   pairs routed to other ranks' experts and writes each token's slot-ordered
   partial sum over this rank's pairs (0 for tokens with none);
4. combine: reduce-scatter (sum) of the [P*T, H] partials, so that each rank
   receives the sum of the P partials of its own home tokens.

Two implementations of steps 2 and 4 share the compute step:

* "p2p" (default on GPUs, `PeerExchange`): the library's own kernels write
  the home rows and the partials straight into the other GPUs' memory over
  NVLink (CUDA IPC mappings of each rank's exchange slab) and signal with
  system-scope counters (mrml_moe_ep_dispatch / mrml_moe_ep_combine); the
  home rank sums the N partials of its tokens in rank order;
* "nccl" (`ep_exchange`): all-gathers and a reduce-scatter through
  torch.distributed (gloo in the CPU tests).  Without a host round trip for
  per-peer counts, an all-to-all has to move fixed-capacity buffers, and a
  capacity of T rows per peer is exactly what the all-gather moves.

Neither needs host synchronisation, so a whole step can be captured into
one CUDA graph.

Numerics: each shard's partial is computed bit for bit as the single-device
path computes it with the other experts' weights set to zero (the Q8_0
quantisation of a row does not depend on which rank does it).  Summing the
P partials replaces the single-device slot-ordered sum, so the layer output
equals the reference within rounding (exactly, for P = 2, where a sum of two
terms does not depend on order).

The compute step is injectable (`shard_fn`), so the orchestration is tested
on CPU ranks with the oracle standing in for the library.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

# shard_fn(x_all [P*T, H] f32, ids_all [P*T, K] i32, probs_all [P*T, K] f32, out [P*T, H] f32) -> None
ShardFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], None]


def shard_range(rank: int, world: int, n_experts: int) -> Tuple[int, int]:
    """(first expert, expert count) of `rank`: contiguous, equal blocks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_experts % world != 0:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    per = n_experts // world
    return rank * per, per


class ExchangeBuffers:
    """Device buffers of one expert-parallel step, allocated once so that the
    step can be replayed from a CUDA graph."""

    def __init__(self, world: int, T: int, H: int, K: int, device):
        self.world, self.T, self.H, self.K = world, T, H, K
        n = world * T
        self.x_all = torch.empty((n, H), dtype=torch.float32, device=device)
        self.ids_all = torch.empty((n, K), dtype=torch.int32, device=device)
        self.probs_all = torch.empty((n, K), dtype=torch.float32, device=device)
        self.partial = torch.empty((n, H), dtype=torch.float32, device=device)


def _all_gather_3(bufs: ExchangeBuffers, x, ids, probs, group) -> None:
    """The three dispatch all-gathers, issued as one NCCL group (one launch)
    where the backend supports coalescing, else one after another."""
    cm = getattr(dist, "_coalescing_manager", None)
    if cm is not None and x.is_cuda:
        with cm(group=group, device=x.device):
            dist.all_gather_into_tensor(bufs.x_all, x, group=group)
            dist.all_gather_into_tensor(bufs.ids_all, ids, group=group)
            dist.all_gather_into_tensor(bufs.probs_all, probs, group=group)
        return
    dist.all_gather_into_tensor(bufs.x_all, x, group=group)
    dist.all_gather_into_tensor(bufs.ids_all, ids, group=group)
    dist.all_gather_into_tensor(bufs.probs_all, probs, group=group)


def ep_exchange(bufs: ExchangeBuffers, x_home: torch.Tensor, ids_home: torch.Tensor, probs_home: torch.Tensor,
                shard_fn: ShardFn, out_home: torch.Tensor, group=None) -> torch.Tensor:
    """Steps 2-4 for this rank's routed home tokens; writes and returns
    out_home [T, H].  Every rank calls it with the same T (the collectives
    are the same on every rank, in the same order)."""
    T, K = ids_home.shape
    if x_home.shape != (bufs.T, bufs.H) or T != bufs.T or K != bufs.K:
        raise ValueError("home batch does not match the exchange buffers")
    if bufs.world == 1:
        shard_fn(x_home, ids_home, probs_home, out_home)
        return out_home
    _all_gather_3(bufs, x_home.contiguous(), ids_home.contiguous(), probs_home.contiguous(), group)
    shard_fn(bufs.x_all, bufs.ids_all, bufs.probs_all, bufs.partial)
    dist.reduce_scatter_tensor(out_home, bufs.partial, op=dist.ReduceOp.SUM, group=group)
    return out_home


class PeerExchange:
    """This rank's exchange slab, the other ranks' slabs mapped over CUDA IPC,
    and the contiguous buffers the experts read (mrml_moe_ep_dispatch /
    mrml_moe_ep_combine).  Set-up is collective: every rank of `group`
    constructs it with the same shapes.  close() is collective too."""

    def __init__(self, moe, rank: int, world: int, T: int, H: int, K: int, device, status, group=None):
        self.moe, self.rank, self.world, self.group = moe, rank, world, group
        self.T, self.H, self.K = T, H, K
        self.status = status  # int32 device word(s) that receive a timeout code
        self.bufs = ExchangeBuffers(world, T, H, K, device)
        self.own = moe.ep_slab_alloc(world, T, H, K)
        handles = [None] * world
        dist.all_gather_object(handles, moe.ipc_get_handle(self.own), group=group)
        self.opened = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self.own)
            else:
                p = moe.ipc_open_handle(handles[r])
                self.opened.append(p)
                ptrs.append(p)
        self.slabs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def exchange(self, x_home, ids_home, probs_home, shard_fn: ShardFn, out_home):
        m, b = self.moe, self.bufs
        args = (self.slabs, self.rank, self.world, self.T, self.H, self.K)
        m.ep_dispatch(*args, x_home, ids_home, probs_home, b.x_all, b.ids_all, b.probs_all, self.status)
        shard_fn(b.x_all, b.ids_all, b.probs_all, b.partial)
        m.ep_combine(*args, b.partial, out_home, self.status)
        return out_home

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            self.moe.ipc_close_handle(p)
        self.opened = []
        dist.barrier(group=self.group)
        if self.own:
            self.moe.ep_slab_free(self.own)
            self.own = 0


class ExpertParallelLayer:
    """One MoE layer (router replicated, experts sharded) on this rank's GPU,
    through the library's C ABI.

    gate_up / down hold this rank's experts only (shard_range), in the GGUF
    layout of mrml_moe_experts; router_w is the full [E, H] router."""

    def __init__(self, moe, rank: int, world: int, wtype: int, H: int, I: int, E: int, K: int, T: int, device,
                 group=None, exchange: str = "p2p"):
        self.moe, self.rank, self.world, self.group = moe, rank, world, group
        self.wtype, self.H, self.I, self.E, self.K, self.T = wtype, H, I, E, K, T
        self.first, self.count = shard_range(rank, world, E)
        self.logits = torch.empty((T, E), dtype=torch.float32, device=device)
        self.ids = torch.empty((T, K), dtype=torch.int32, device=device)
        self.probs = torch.empty((T, K), dtype=torch.float32, device=device)
        self.router_ws = moe.new_workspace(H, I, E, K, T, device)
        self.ws = moe.new_workspace(H, I, self.count, K, world * T, device)
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.exchange = exchange if world > 1 else "nccl"
        if self.exchange == "p2p":
            self.peer = PeerExchange(moe, rank, world, T, H, K, device, self.ws, group)
            self.bufs = self.peer.bufs
        else:
            self.peer = None
            self.bufs = ExchangeBuffers(world, T, H, K, device)

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def forward(self, router_w, x_home, gate_up, down, out_home, down_scale: Optional[torch.Tensor] = None):
        m = self.moe
        m.router(router_w, x_home, self.logits, self.ids, self.probs, self.H, self.E, self.K, self.T, self.router_ws)

        def shard_fn(x, ids, probs, out):
            m.experts_shard(self.wtype, gate_up, down, ids, probs, down_scale, x, out, self.H, self.I, self.E,
                            self.first, self.count, self.K, x.shape[0], self.ws)

        if self.peer is not None:
            return self.peer.exchange(x_home, self.ids, self.probs, shard_fn, out_home)
        return ep_exchange(self.bufs, x_home, self.ids, self.probs, shard_fn, out_home, self.group)
