"""Expert-parallel shards on the GPU.

* mrml_moe_experts_shard on one GPU, on each expert-product path: every
  shard's partial equals, bit for bit, both the single-device
  mrml_moe_experts call and the oracle with the other shards' pairs given
  weight 0; the partials add up to the layer within tolerance.
* The expert-parallel layer on 2 GPUs (NCCL all-gather / reduce-scatter),
  when the box has them: equal to the sum of the two shards' partials bit
  for bit, and to the reference within tolerance.
"""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from test_ep import _case, oracle_shard, synth_range
from test_gpu_parity import PATHS, assert_close, assert_exact, dev_tensor

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(params=sorted(PATHS))
def expert_path(request, cuda, moe):
    moe.set_expert_path(PATHS[request.param])
    yield request.param
    moe.set_expert_path(0)


def _gpu_case(synth, oracle, moe, device, wtype, H, I, E, K, T, seed):
    """Like test_ep._case, with the expert weights generated and quantised on
    the GPU (the quantiser is byte-exact to the reference's)."""
    gu, dn = synth.expert_weights_device(seed, wtype, H, I, E, device, moe.quantize)
    W = synth.normal(seed + 1000, E * H, 0.02).reshape(E, H)
    x = synth.normal(seed + 77, T * H).reshape(T, H)
    _, ids, probs = oracle.router(W, x, H, E, K, T)
    return gu.cpu().numpy(), dn.cpu().numpy(), ids, probs, x


def _shard_on_gpu(moe, device, wtype, gu, dn, ids, probs, scale, x, H, I, E, first, count, K):
    import torch

    T = x.shape[0]
    gu_e = gu.reshape(E, -1)[first:first + count]
    dn_e = dn.reshape(E, -1)[first:first + count]
    out = torch.full((T, H), float("nan"), device=device)
    ws = moe.new_workspace(H, I, count, K, T, device)
    moe.experts_shard(wtype, dev_tensor(gu_e, device), dev_tensor(dn_e, device), dev_tensor(ids, device),
                      dev_tensor(probs, device), None if scale is None else dev_tensor(scale, device),
                      dev_tensor(x, device), out, H, I, E, first, count, K, T, ws)
    st, _ = moe.device_status(ws)
    assert st == 0, f"device status {st}"
    return out.cpu().numpy()


_ORACLE = {}


def _masked_on_gpu(moe, device, wtype, gu, dn, ids, probs, x, H, I, E, first, count, K):
    """The single-device layer with the pairs outside [first, first+count)
    given weight 0."""
    import torch

    T = x.shape[0]
    loc = (ids >= first) & (ids < first + count)
    out = torch.full((T, H), float("nan"), device=device)
    ws = moe.new_workspace(H, I, E, K, T, device)
    moe.experts(wtype, dev_tensor(gu, device), dev_tensor(dn, device), dev_tensor(ids, device),
                dev_tensor(np.where(loc, probs, 0).astype(np.float32), device), None, dev_tensor(x, device), out, H,
                I, E, K, T, ws)
    st, _ = moe.device_status(ws)
    assert st == 0, f"device status {st}"
    return out.cpu().numpy()


# (2, 2816, 704, 128, 8, 256): the expert-parallel decode shape at N = 4..8
# (256+ tokens per shard call: the per-token quantisation and group gather,
# and 16-position units from 12 pairs per expert).
@pytest.mark.parametrize("wtype,H,I,E,K,T", [(2, 2816, 704, 128, 8, 64), (8, 1024, 512, 16, 2, 300),
                                              (2, 256, 128, 8, 3, 7), (2, 2816, 704, 128, 8, 256)])
def test_experts_shard_bit_exact(cuda, moe, oracle, synth, expert_path, wtype, H, I, E, K, T):
    key = (wtype, H, I, E, K, T)
    if key not in _ORACLE:  # the oracle's answers are shared by the three paths
        gu, dn, ids, probs, x = _gpu_case(synth, oracle, moe, cuda, wtype, H, I, E, K, T, 21)
        ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, T, os.cpu_count() or 1)
        parts = {}
        for world in (2, 8):
            for r in range(world):
                first, count = synth_range(r, world, E)
                parts[world, r] = oracle_shard(oracle, wtype, gu, dn, first, count, H, I, E, K)(x, ids, probs)
        _ORACLE[key] = (gu, dn, ids, probs, x, ref, parts)
    gu, dn, ids, probs, x, ref, parts = _ORACLE[key]
    for world in (2, 8):
        total = np.zeros_like(ref)
        for r in range(world):
            first, count = synth_range(r, world, E)
            got = _shard_on_gpu(moe, cuda, wtype, gu, dn, ids, probs, None, x, H, I, E, first, count, K)
            same = _masked_on_gpu(moe, cuda, wtype, gu, dn, ids, probs, x, H, I, E, first, count, K)
            assert np.array_equal(got, same), f"shard {r}/{world}: {np.count_nonzero(got != same)} elements differ"
            assert_exact(got, parts[world, r])
            total += got
        assert_close(total, ref)


def test_experts_shard_scale_uses_global_ids(cuda, moe, oracle, synth):
    wtype, H, I, E, K, T = 8, 256, 128, 8, 2, 9
    gu, dn, ids, probs, x = _case(synth, oracle, wtype, H, I, E, K, T, 3)
    scale = (0.5 + np.arange(E, dtype=np.float32) / 4).astype(np.float32)
    ref = oracle.experts(wtype, gu, dn, ids, probs, scale, x, H, I, E, K, T)
    a = _shard_on_gpu(moe, cuda, wtype, gu, dn, ids, probs, scale, x, H, I, E, 0, 4, K)
    b = _shard_on_gpu(moe, cuda, wtype, gu, dn, ids, probs, scale, x, H, I, E, 4, 4, K)
    assert np.isfinite(a).all() and np.isfinite(b).all()
    assert_close(a + b, ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, args, exchange, results):
    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from tests.conftest import _load

    moe = _load("mrml_moe_b200", os.path.join(ROOT, "qt_llama.cpp_b200", "mrml_moe.py"))
    synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
    ep = _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))
    wtype, H, I, E, K, T, seed, steps = args
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    layer = None
    try:
        gu, dn = synth.expert_weights_device(seed, wtype, H, I, E, dev, moe.quantize)
        W = dev_tensor(synth.normal(seed + 1000, E * H, 0.02).reshape(E, H), dev)
        layer = ep.ExpertParallelLayer(moe, rank, world, wtype, H, I, E, K, T, dev, exchange=exchange)
        f, c = layer.first, layer.count
        gu_l = gu[f:f + c].contiguous()
        dn_l = dn[f:f + c].contiguous()
        del gu, dn
        x_in = torch.empty((T, H), device=dev)
        out = torch.empty((T, H), device=dev)
        outs, idss = [], []
        # The first half of the steps eager, the rest replayed from one CUDA
        # graph with new inputs copied into its input buffer.
        graph = None
        for s in range(steps):
            x = synth.normal(seed + 77 + s, world * T * H).reshape(world * T, H)
            x_in.copy_(torch.from_numpy(x[rank * T:(rank + 1) * T]))
            if s < steps // 2:
                layer.forward(W, x_in, gu_l, dn_l, out)
            else:
                if graph is None:
                    graph = torch.cuda.CUDAGraph()
                    side = torch.cuda.Stream(device=dev)
                    side.wait_stream(torch.cuda.current_stream())
                    torch.cuda.synchronize()
                    with torch.cuda.graph(graph, stream=side):
                        layer.forward(W, x_in, gu_l, dn_l, out)
                graph.replay()
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy().copy())
            idss.append(layer.ids.cpu().numpy().copy())
        del graph
        st, _ = moe.device_status(layer.ws)
        results.put((rank, outs, idss, st))
    except Exception as exc:
        results.put((rank, repr(exc), None, None))
    finally:
        if layer is not None:
            try:
                layer.close()
            except Exception:
                pass
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_ep_layer_two_gpus(cuda, moe, oracle, synth, exchange):
    """Four consecutive layer steps (two eager, two replayed from a CUDA
    graph) on 2 GPUs: every output equals the sum of the two shards'
    partials bit for bit, and the reference within tolerance."""
    import multiprocessing as mp

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world, steps = 2, 4
    args = (2, 2816, 704, 128, 8, 32, 9, steps)
    wtype, H, I, E, K, T, seed, _ = args
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, args, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, outs, idss, st = q.get(timeout=300)
            assert not isinstance(outs, str), f"rank {r}: {outs}"
            assert st == 0
            got[r] = (outs, idss)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    gu_d, dn_d = synth.expert_weights_device(seed, wtype, H, I, E, cuda, moe.quantize)
    gu, dn = gu_d.cpu().numpy(), dn_d.cpu().numpy()
    W = synth.normal(seed + 1000, E * H, 0.02).reshape(E, H)
    for s in range(steps):
        x = synth.normal(seed + 77 + s, world * T * H).reshape(world * T, H)
        _, ids, probs = oracle.router(W, x, H, E, K, world * T)
        parts = [_shard_on_gpu(moe, cuda, wtype, gu, dn, ids, probs, None, x, H, I, E, *synth_range(r, world, E), K)
                 for r in range(world)]
        ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, world * T, os.cpu_count() or 1)
        for r in range(world):
            outs, idss = got[r]
            home = slice(r * T, (r + 1) * T)
            np.testing.assert_array_equal(idss[s], ids[home])
            np.testing.assert_array_equal(outs[s], parts[0][home] + parts[1][home])
            assert_close(outs[s], ref[home])


# --------------------------------------------- the peer exchange, one GPU
# The N ranks of the peer exchange are emulated on one GPU: N slabs in this
# GPU's memory, and each rank's calls issued in an order in which every wait
# is already satisfied by kernels that completed earlier on the same stream
# (all dispatches, then all expert steps, then all combines), so no kernel
# ever waits on a kernel that runs at the same time.


def _ep_module():
    from tests.conftest import _load

    return _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))


class OneGpuRanks:
    """N emulated ranks' slabs, workspaces and expert shards on cuda:0."""

    def __init__(self, moe, device, N, wtype, gu, dn, H, I, E, K, T, packed=False):
        import torch

        self.moe, self.N, self.H, self.I, self.E, self.K, self.T = moe, N, H, I, E, K, T
        self.wcall = wtype | (moe.MRML_PACKED if packed else 0)
        self.own = [moe.ep_slab_alloc(N, T, H, K) for _ in range(N)]
        self.slabs = torch.tensor(self.own, dtype=torch.int64, device=device)
        self.ws = [moe.new_ep_workspace(N, T, H, I, E, K, device) for _ in range(N)]
        per = E // N
        self.w = []
        for r in range(N):
            g = dev_tensor(gu.reshape(E, -1)[r * per:(r + 1) * per], device)
            d = dev_tensor(dn.reshape(E, -1)[r * per:(r + 1) * per], device)
            if packed:
                g, d = moe.prepare_weights(wtype, g.reshape(per, 2 * I, -1), d.reshape(per, H, -1))
            self.w.append((g, d))

    def step(self, x, ids, probs, out):
        m, N, H, E, K, T = self.moe, self.N, self.H, self.E, self.K, self.T
        for r in range(N):
            m.ep_dispatch(self.slabs, r, N, T, H, E, K, x[r], ids[r], probs[r])
        for r in range(N):
            m.ep_experts(self.wcall, self.w[r][0], self.w[r][1], None, self.slabs, r, N, T, H, self.I, E, K,
                         self.ws[r])
        for r in range(N):
            m.ep_combine(self.slabs, r, N, T, H, E, K, ids[r], probs[r], out[r], self.ws[r])

    def close(self):
        import torch

        torch.cuda.synchronize()
        for p in self.own:
            self.moe.ep_slab_free(p)
        self.own = []


@pytest.mark.parametrize("N,wtype,H,I,E,K,T,packed", [(2, 2, 2816, 704, 128, 8, 16, False),
                                                       (4, 8, 1024, 512, 16, 2, 40, False),
                                                       (8, 2, 2816, 704, 128, 8, 8, True)])
def test_peer_exchange_one_gpu(cuda, moe, oracle, synth, N, wtype, H, I, E, K, T, packed):
    """Two consecutive steps of the sparse peer exchange with N ranks on one
    GPU: every rank's output equals, bit for bit, the rank-ordered sum of
    the oracle shards' partials over the ranks that own the token's experts,
    and the reference within tolerance."""
    import torch

    ep = _ep_module()
    gu_d, dn_d = synth.expert_weights_device(31 + N, wtype, H, I, E, cuda, moe.quantize)
    gu, dn = gu_d.cpu().numpy(), dn_d.cpu().numpy()
    del gu_d, dn_d
    W = synth.normal(32 + N, E * H, 0.02).reshape(E, H)
    R = OneGpuRanks(moe, cuda, N, wtype, gu, dn, H, I, E, K, T, packed)
    try:
        for step in range(2):
            x = synth.normal(40 + 10 * N + step, N * T * H).reshape(N * T, H)
            _, ids, probs = oracle.router(W, x, H, E, K, N * T)
            xs = [dev_tensor(x[r * T:(r + 1) * T], cuda) for r in range(N)]
            idd = [dev_tensor(ids[r * T:(r + 1) * T], cuda) for r in range(N)]
            prd = [dev_tensor(probs[r * T:(r + 1) * T], cuda) for r in range(N)]
            outs = [torch.full((T, H), float("nan"), device=cuda) for _ in range(N)]
            R.step(xs, idd, prd, outs)
            for r in range(N):
                assert moe.device_status(R.ws[r])[0] == 0
            parts = [oracle_shard(oracle, wtype, gu, dn, *synth_range(q, N, E), H, I, E, K)(x, ids, probs)
                     for q in range(N)]
            want = ep.sparse_sum(parts, ep.owner_masks(ids, probs, N, E))
            ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, N * T, os.cpu_count() or 1)
            for r in range(N):
                home = slice(r * T, (r + 1) * T)
                got = outs[r].cpu().numpy()
                assert_exact(got, want[home])
                assert_close(got, ref[home])
    finally:
        R.close()


def test_peer_exchange_wait_times_out(cuda, moe, synth):
    """A rank whose peer never pushes: with a short spin limit the receive
    wait and the combine wait give up, the device status reads
    MRML_ERR_DEVICE_TIMEOUT, and the output is left untouched.  The wait is
    bounded and returns; nothing hangs."""
    import torch

    N, wtype, H, I, E, K, T = 2, 2, 256, 128, 8, 2, 4
    gu, dn = synth.expert_weights(51, wtype, H, I, E)
    R = OneGpuRanks(moe, cuda, N, wtype, gu, dn, H, I, E, K, T)
    moe.set_exchange_spin_limit(1 << 12)
    try:
        x = dev_tensor(synth.normal(52, T * H).reshape(T, H), cuda)
        ids = dev_tensor(np.array([[0, 5], [1, 6], [2, 7], [3, 4]], np.int32), cuda)
        probs = dev_tensor(np.full((T, K), 0.5, np.float32), cuda)
        out = torch.full((T, H), 7.0, device=cuda)
        # rank 0 alone: rank 1 never dispatches nor combines
        moe.ep_dispatch(R.slabs, 0, N, T, H, E, K, x, ids, probs)
        moe.ep_experts(R.wcall, R.w[0][0], R.w[0][1], None, R.slabs, 0, N, T, H, I, E, K, R.ws[0])
        moe.ep_combine(R.slabs, 0, N, T, H, E, K, ids, probs, out, R.ws[0])
        st, _ = moe.device_status(R.ws[0])
        assert st == -6  # MRML_ERR_DEVICE_TIMEOUT
        assert torch.all(out == 7.0)
        assert moe.device_status(R.ws[0])[0] == 0  # reading clears it
    finally:
        moe.set_exchange_spin_limit(0)
        R.close()
