"""Expert parallelism for the MoE layer across the GPUs of one node.

The reference runs the whole layer on one device (its MoE call is
CudaDevice::moe_topk_batch_q4_0, crates/mrml-tensor/src/cuda.rs:2840-2880,
and nothing in it communicates).  Here the experts are sharded: rank r of N
holds the contiguous experts [r*E/N, (r+1)*E/N) and owns T "home" tokens.
One layer step on every rank:

1. route the home tokens with the replicated router (mrml_moe_router);
2. dispatch: quantise each home row to Q8_0 once and send it only to the
   ranks that own one of its experts (with every home token's ids and
   weights);
3. compute: this rank's experts on the rows it received;
4. combine: each rank returns, per received token, the slot-ordered partial
   sum over its own pairs to the token's home rank, which adds the partials
   of the ranks that own its experts in rank order.

Two implementations of steps 2-4:

* "p2p" (default on GPUs, `PeerExchange`): the library's own kernels store
  the rows and the partials straight into the other GPUs' memory over NVLink
  (CUDA IPC mappings of each rank's exchange slab) and signal with
  system-scope counters: mrml_moe_ep_dispatch, mrml_moe_ep_experts,
  mrml_moe_ep_combine.  Sparse: bytes cross NVLink only for (token, rank)
  pairs where the rank owns one of the token's experts;
* "nccl" (`ep_exchange`): all-gathers of the home rows, ids and weights and a
  reduce-scatter of dense [N*T, H] partials through torch.distributed (gloo
  in the CPU tests), with mrml_moe_experts_shard as the compute.  Without a
  host round trip for per-peer counts an all-to-all must move fixed-capacity
  buffers, so this dense form is the collective-library baseline.

Neither needs host synchronisation, so a whole step can be captured into
one CUDA graph.

Numerics: each rank's partial is the single-device slot-ordered sum
restricted to its pairs, computed bit for bit as the single-device path
computes it (the Q8_0 quantisation of a row does not depend on which rank
does it).  The home rank adds the partials in rank order (`sparse_sum`), so
the layer output equals the reference within rounding, and exactly for a
token whose experts all sit on one rank.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import numpy as np
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


def owner_masks(ids: np.ndarray, probs: np.ndarray, world: int, n_experts: int) -> np.ndarray:
    """[T, world] bool: rank q owns one of token t's experts (pairs with
    weight > 1e-4 and an id in range), i.e. t's row is sent to q and q sends a
    partial back."""
    per = n_experts // world
    ids = np.asarray(ids)
    ok = (np.asarray(probs) > np.float32(1e-4)) & (ids >= 0) & (ids < n_experts)
    owner = np.where(ok, ids // per, -1)
    return np.stack([(owner == q).any(axis=1) for q in range(world)], axis=1)


def sparse_sum(partials, masks: np.ndarray) -> np.ndarray:
    """The home rank's reduce: per token, the partials of the ranks in its
    mask added in rank order (f32, the first term taken as is), 0 without
    any.  partials: [world] arrays [T, H]."""
    T, H = partials[0].shape
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        first = True
        for q in range(masks.shape[1]):
            if not masks[t, q]:
                continue
            if first:
                out[t] = partials[q][t]
                first = False
            else:
                out[t] = (out[t] + partials[q][t]).astype(np.float32)
    return out


def exchange_bytes(ids: np.ndarray, probs: np.ndarray, world: int, n_experts: int, H: int, K: int, rank: int,
                   T: int) -> dict:
    """Bytes rank `rank` receives over NVLink in one step of the p2p exchange
    (from the other ranks only): dispatch = Q8_0 rows (H values + H/32 f16
    scales) of the tokens routed here plus every rank's ids and weights;
    combine = f32 partial rows of this rank's home tokens from the other
    ranks that own one of their experts.  ids/probs: all ranks' [world*T, K]
    in rank order."""
    masks = owner_masks(ids, probs, world, n_experts)
    row = H + (H // 32) * 2
    disp = 0
    for src in range(world):
        if src == rank:
            continue
        disp += int(masks[src * T:(src + 1) * T, rank].sum()) * row + T * K * 8
    home = masks[rank * T:(rank + 1) * T]
    comb = int(sum(home[:, q].sum() for q in range(world) if q != rank)) * H * 4
    return {"dispatch": disp, "combine": comb, "total": disp + comb}


class ExchangeBuffers:
    """Device buffers of one NCCL-baseline step, allocated once so that the
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
    """The NCCL baseline's steps 2-4 for this rank's routed home tokens;
    writes and returns out_home [T, H].  Every rank calls it with the same T
    (the collectives are the same on every rank, in the same order)."""
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
    """This rank's exchange slab and the other ranks' slabs mapped over CUDA
    IPC (the device array `slabs`, rank order).  Set-up is collective: every
    rank of `group` constructs it with the same shapes.  close() is collective
    too."""

    def __init__(self, moe, rank: int, world: int, T: int, H: int, K: int, device, group=None):
        self.moe, self.rank, self.world, self.group = moe, rank, world, group
        self.T, self.H, self.K = T, H, K
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

    gate_up / down hold this rank's experts only (shard_range), in the layout
    of mrml_moe_experts (GGUF, or packed with wtype | MRML_PACKED); router_w
    is the full [E, H] router."""

    def __init__(self, moe, rank: int, world: int, wtype: int, H: int, I: int, E: int, K: int, T: int, device,
                 group=None, exchange: str = "p2p"):
        self.moe, self.rank, self.world, self.group = moe, rank, world, group
        self.wtype, self.H, self.I, self.E, self.K, self.T = wtype, H, I, E, K, T
        self.first, self.count = shard_range(rank, world, E)
        self.logits = torch.empty((T, E), dtype=torch.float32, device=device)
        self.ids = torch.empty((T, K), dtype=torch.int32, device=device)
        self.probs = torch.empty((T, K), dtype=torch.float32, device=device)
        self.router_ws = moe.new_workspace(H, I, E, K, T, device)
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.exchange = exchange if world > 1 else "nccl"
        if self.exchange == "p2p":
            self.peer = PeerExchange(moe, rank, world, T, H, K, device, group)
            self.ws = moe.new_ep_workspace(world, T, H, I, E, K, device)
            self.bufs = None
        else:
            self.peer = None
            self.ws = moe.new_workspace(H, I, self.count, K, world * T, device)
            self.bufs = ExchangeBuffers(world, T, H, K, device)

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def forward(self, router_w, x_home, gate_up, down, out_home, down_scale: Optional[torch.Tensor] = None,
                router_x: Optional[torch.Tensor] = None):
        """One layer step; router_x is the router's input (model.rs:1774-1784)
        when it differs from the experts' input x_home."""
        m = self.moe
        m.router(router_w, x_home if router_x is None else router_x, self.logits, self.ids, self.probs, self.H,
                 self.E, self.K, self.T, self.router_ws)
        if self.peer is not None:
            args = (self.peer.slabs, self.rank, self.world, self.T, self.H)
            m.ep_dispatch(*args, self.E, self.K, x_home, self.ids, self.probs)
            m.ep_experts(self.wtype, gate_up, down, down_scale, *args, self.I, self.E, self.K, self.ws)
            m.ep_combine(*args, self.E, self.K, self.ids, self.probs, out_home, self.ws)
            return out_home

        def shard_fn(x, ids, probs, out):
            m.experts_shard(self.wtype, gate_up, down, ids, probs, down_scale, x, out, self.H, self.I, self.E,
                            self.first, self.count, self.K, x.shape[0], self.ws)

        return ep_exchange(self.bufs, x_home, self.ids, self.probs, shard_fn, out_home, self.group)
