"""Expert-parallel orchestration on CPU ranks (gloo), with the oracle as the
per-shard compute.  The GPU runs the same ep_exchange with the library's
mrml_moe_experts_shard and NCCL."""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(synth, oracle, wtype, H, I, E, K, T_all, seed):
    gu, dn = synth.expert_weights(seed, wtype, H, I, E)
    W = synth.normal(seed + 1000, E * H, 0.02).reshape(E, H)
    x = synth.normal(seed + 77, T_all * H).reshape(T_all, H)
    _, ids, probs = oracle.router(W, x, H, E, K, T_all)
    return gu, dn, ids, probs, x


def oracle_shard(oracle, wtype, gu, dn, first, count, H, I, E, K):
    """The shard's partial: the oracle's layer with the pairs of other
    shards' experts given weight 0 (skipped by the alpha <= 1e-4 rule)."""
    gu_e = gu.reshape(E, -1)[first:first + count]
    dn_e = dn.reshape(E, -1)[first:first + count]

    def fn(x, ids, probs):
        loc = (ids >= first) & (ids < first + count)
        ids_l = np.where(loc, ids - first, 0).astype(np.int32)
        probs_l = np.where(loc, probs, 0).astype(np.float32)
        return oracle.experts(wtype, gu_e, dn_e, ids_l, probs_l, None, x, H, I, count, K, x.shape[0],
                              os.cpu_count() or 1)

    return fn


def _worker(rank, world, port, args, results):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from tests.conftest import _load

    synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
    oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    ep = _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))
    wtype, H, I, E, K, T, seed = args
    import datetime

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        gu, dn, ids, probs, x = _case(synth, oracle, wtype, H, I, E, K, world * T, seed)
        first, count = ep.shard_range(rank, world, E)
        fn = oracle_shard(oracle, wtype, gu, dn, first, count, H, I, E, K)
        home = slice(rank * T, (rank + 1) * T)

        def shard_fn(xa, ia, pa, out):
            out.copy_(torch.from_numpy(fn(xa.numpy(), ia.numpy(), pa.numpy())))

        bufs = ep.ExchangeBuffers(world, T, H, K, "cpu")
        out = torch.empty((T, H), dtype=torch.float32)
        ep.ep_exchange(bufs, torch.from_numpy(x[home]), torch.from_numpy(ids[home]), torch.from_numpy(probs[home]),
                       shard_fn, out)
        results.put((rank, out.numpy().copy(), bufs.ids_all.numpy().copy()))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, repr(exc), None))
    finally:
        dist.destroy_process_group()


def _run_ranks(world, args):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, out, ids_all = q.get(timeout=180)
            assert not isinstance(out, str), f"rank {r}: {out}"
            got[r] = (out, ids_all)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return got


@pytest.mark.parametrize("world", [2, 4])
def test_ep_matches_single_device(world, synth, oracle):
    wtype, H, I, E, K, T, seed = 8, 256, 128, 8, 2, 3, 11
    got = _run_ranks(world, (wtype, H, I, E, K, T, seed))
    gu, dn, ids, probs, x = _case(synth, oracle, wtype, H, I, E, K, world * T, seed)
    ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, world * T)
    parts = [oracle_shard(oracle, wtype, gu, dn, *synth_range(r, world, E), H, I, E, K)(x, ids, probs)
             for r in range(world)]
    for r in range(world):
        out, ids_all = got[r]
        np.testing.assert_array_equal(ids_all, ids)  # the dispatch saw every rank's routing
        home = slice(r * T, (r + 1) * T)
        err = np.abs(out - ref[home]).max()
        assert err <= 1e-3 * np.abs(ref).max()
        assert np.linalg.norm(out - ref[home]) <= 1e-4 * np.linalg.norm(ref[home])
        if world == 2:  # a two-term sum does not depend on order: exact
            np.testing.assert_array_equal(out, parts[0][home] + parts[1][home])


def synth_range(rank, world, E):
    per = E // world
    return rank * per, per


def test_shard_partials_sum_to_layer(synth, oracle):
    """Single process: the shards' partials add up to the layer (the
    property the reduce-scatter relies on), and a one-shard split is the
    layer itself, bit for bit."""
    wtype, H, I, E, K, T = 2, 256, 128, 8, 3, 6
    gu, dn, ids, probs, x = _case(synth, oracle, wtype, H, I, E, K, T, 5)
    ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, T)
    whole = oracle_shard(oracle, wtype, gu, dn, 0, E, H, I, E, K)(x, ids, probs)
    np.testing.assert_array_equal(whole, ref)
    for world in (2, 4, 8):
        s = sum(oracle_shard(oracle, wtype, gu, dn, *synth_range(r, world, E), H, I, E, K)(x, ids, probs)
                for r in range(world))
        assert np.abs(s - ref).max() <= 1e-3 * np.abs(ref).max()
        assert np.linalg.norm(s - ref) <= 1e-4 * np.linalg.norm(ref)


def test_shard_range():
    sys.path.insert(0, ROOT)
    from tests.conftest import _load

    ep = _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))
    assert ep.shard_range(0, 8, 128) == (0, 16)
    assert ep.shard_range(7, 8, 128) == (112, 16)
    with pytest.raises(ValueError):
        ep.shard_range(0, 3, 128)
    with pytest.raises(ValueError):
        ep.shard_range(2, 2, 128)


def _ep_module():
    sys.path.insert(0, ROOT)
    from tests.conftest import _load

    return _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sparse_exchange_semantics(world, synth, oracle):
    """The peer exchange's arithmetic, restated on the host: each rank's
    partial is the oracle shard; the home rank adds the partials of the
    ranks that own the token's experts in rank order.  Within the layer
    tolerance of the reference, and equal to it bit for bit for tokens whose
    experts all sit on one rank."""
    ep = _ep_module()
    wtype, H, I, E, K, T = 2, 256, 128, 16, 4, 24
    gu, dn, ids, probs, x = _case(synth, oracle, wtype, H, I, E, K, T, 13)
    probs[3, 1] = 0.0  # a skipped slot does not make its rank an owner
    ref = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, E, K, T)
    parts = [oracle_shard(oracle, wtype, gu, dn, *synth_range(r, world, E), H, I, E, K)(x, ids, probs)
             for r in range(world)]
    masks = ep.owner_masks(ids, probs, world, E)
    assert masks.shape == (T, world) and masks.any(axis=1).all()
    if world > 1:
        per = E // world
        assert not masks[3, ids[3, 1] // per] or ((ids[3] // per == ids[3, 1] // per) & (probs[3] > 1e-4)).any()
    out = ep.sparse_sum(parts, masks)
    assert np.abs(out - ref).max() <= 1e-3 * np.abs(ref).max()
    assert np.linalg.norm(out - ref) <= 1e-4 * np.linalg.norm(ref)
    single = masks.sum(axis=1) == 1
    np.testing.assert_array_equal(out[single], ref[single])
    # bytes: every received row is counted once per (token, receiving rank)
    b = ep.exchange_bytes(np.tile(ids, (world, 1)), np.tile(probs, (world, 1)), world, E, H, K, 0, T)
    row = H + H // 32 * 2
    assert b["dispatch"] == (world - 1) * (int(masks[:, 0].sum()) * row + T * K * 8)
    assert b["combine"] == int(masks[:, 1:].sum()) * H * 4
