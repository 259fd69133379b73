"""Parity of the fused FFN prologue / epilogue and the shared dense MLP with
the reference's CPU layer (model.rs:1719-1784, 2093-2109, 2176-2196).

All three are restatements of f32 arithmetic in the reference's order, so
the bar is bit-identical to the oracle; the whole-layer case chains them with
the MoE forward as a Gemma-4 MoE layer does.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def assert_exact(got, ref):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert got.shape == ref.shape
    diff = got.view(np.uint32) != ref.view(np.uint32)
    assert not diff.any(), f"{np.count_nonzero(diff)} of {diff.size} elements differ (max {np.abs(got - ref).max():.3e})"


def norm_weight(synth, seed, H):
    return (1.0 + synth.normal(seed, H, 0.1)).astype(np.float32)


@pytest.mark.parametrize("H,T,weighted,with_attn", [(2816, 1, True, True), (2816, 64, True, True),
                                                    (2816, 9, False, True), (2816, 5, True, False),
                                                    (1024, 33, True, True), (257, 5, True, True)])
def test_ffn_prologue_bit_exact(cuda, moe, oracle, synth, H, T, weighted, with_attn):
    import torch

    hid = (synth.normal(H * 7 + T, T * H) * 2.5).reshape(T, H)
    attn = (synth.normal(H * 7 + T + 1, T * H) * 0.7).reshape(T, H) if with_attn else None
    ws = [norm_weight(synth, H + i, H) if weighted else None for i in range(4)]
    want = oracle.ffn_prologue(hid, attn, *ws)
    outs = [torch.full((T, H), float("nan"), device=cuda) for _ in range(4)]
    moe.ffn_prologue(dev(hid, cuda), None if attn is None else dev(attn, cuda),
                     *[None if w is None else dev(w, cuda) for w in ws], *outs, H, T)
    for got, ref in zip(outs, want):
        assert_exact(got.cpu().numpy(), ref)


def test_ffn_prologue_optional_outputs(cuda, moe, oracle, synth):
    """A dense layer (no router, no experts) asks for the shared input only;
    the other outputs are left untouched."""
    import torch

    H, T = 2816, 4
    h = synth.normal(5, T * H).reshape(T, H)
    w = norm_weight(synth, 6, H)
    want = oracle.ffn_prologue(h, None, None, w, None, None)[1]
    xs = torch.empty((T, H), device=cuda)
    moe.ffn_prologue(dev(h, cuda), None, None, dev(w, cuda), None, None, None, xs, None, None, H, T)
    assert_exact(xs.cpu().numpy(), want)


def test_reference_surface_prepare_finish(cuda, moe, oracle, synth):
    """MoeDevice.prepare_ffn / finish_ffn (cuda.rs:2914-3016 argument order)
    on one token, as the reference's own GPU test calls them
    (cuda.rs:3340-3420), checked bit for bit against the CPU path."""
    import torch

    H = 2816
    vals = [synth.normal(300 + i, H) for i in range(8)]
    hid, proj = vals[0], vals[1]
    pan, fn, pre, rs, p1, p2 = [(1.0 + 0.1 * v).astype(np.float32) for v in [synth.normal(310 + i, H) for i in range(6)]]
    dense, moe_raw = vals[2], vals[3]
    d = lambda a: dev(a.reshape(1, H), cuda)
    outs = [torch.empty((1, H), device=cuda) for _ in range(4)]
    md = moe.MoeDevice(0)
    md.prepare_ffn(d(hid), d(proj), d(pan), d(fn), d(pre), d(rs), *outs, H)
    want = oracle.ffn_prologue(hid.reshape(1, H), proj.reshape(1, H), pan, fn, pre, rs)
    for got, ref in zip(outs, want):
        assert_exact(got.cpu().numpy(), ref)
    out = torch.empty((1, H), device=cuda)
    md.finish_ffn(outs[0], d(dense), d(moe_raw), d(p1), d(p2), d(pan), out, 0.75, H)
    assert_exact(out.cpu().numpy(), oracle.ffn_epilogue(want[0], dense.reshape(1, H), moe_raw.reshape(1, H), p1, p2,
                                                        pan, 0.75))


@pytest.mark.parametrize("H,T,with_mlp", [(2816, 1, True), (2816, 64, True), (2816, 7, False), (1024, 20, True),
                                          (257, 3, True)])
def test_ffn_epilogue_bit_exact(cuda, moe, oracle, synth, H, T, with_mlp):
    import torch

    attn = synth.normal(11 + T, T * H).reshape(T, H)
    mlp = (synth.normal(12 + T, T * H) * 0.3).reshape(T, H) if with_mlp else None
    moe_raw = (synth.normal(13 + T, T * H) * 0.05).reshape(T, H)
    ws = [norm_weight(synth, 20 + i, H) for i in range(3)]
    scale = np.float32(0.7734375)
    want = oracle.ffn_epilogue(attn, mlp, moe_raw, *ws, float(scale))
    out = torch.full((T, H), float("nan"), device=cuda)
    moe.ffn_epilogue(dev(attn, cuda), None if mlp is None else dev(mlp, cuda), dev(moe_raw, cuda),
                     *[dev(w, cuda) for w in ws], out, float(scale), H, T)
    assert_exact(out.cpu().numpy(), want)
    # in place over the residual, as a layer stack runs it
    d_attn = dev(attn, cuda)
    moe.ffn_epilogue(d_attn, None if mlp is None else dev(mlp, cuda), dev(moe_raw, cuda), *[dev(w, cuda) for w in ws],
                     d_attn, float(scale), H, T)
    assert_exact(d_attn.cpu().numpy(), want)


@pytest.mark.parametrize("wtype,packed,T", [(2, False, 1), (2, True, 1), (2, True, 8), (2, False, 64), (2, True, 64),
                                            (2, True, 200), (8, False, 16)])
def test_dense_ffn_bit_exact(cuda, moe, oracle, synth, wtype, packed, T):
    """The shared dense GeGLU MLP at the reference's sizes (H 2816, I 2112):
    the experts' arithmetic for one expert with weight 1."""
    import torch

    H, I = 2816, 2112
    gu, dn = synth.expert_weights(40 + wtype, wtype, H, I, 1)
    x = synth.normal(41 + T, T * H).reshape(T, H)
    ids = np.zeros((T, 1), np.int32)
    probs = np.ones((T, 1), np.float32)
    want = oracle.experts(wtype, gu, dn, ids, probs, None, x, H, I, 1, 1, T, n_threads=8)
    d_gu, d_dn = dev(gu, cuda), dev(dn, cuda)
    wt = wtype
    if packed:
        d_gu, d_dn = moe.prepare_weights(wtype, d_gu, d_dn)
        wt = wtype | moe.MRML_PACKED
    ws = moe.new_dense_ffn_workspace(H, I, T, cuda)
    out = torch.full((T, H), float("nan"), device=cuda)
    moe.dense_ffn(wt, d_gu, d_dn, dev(x, cuda), out, H, I, T, ws)
    assert_exact(out.cpu().numpy(), want)


@pytest.mark.parametrize("T", [1, 8, 48])
def test_ffn_layer_chain_bit_exact(cuda, moe, oracle, synth, T):
    """One MoE layer's FFN half as the reference runs it (model.rs:1743-2196):
    prologue -> router + top-8 + experts on x_moe, dense MLP on x_shared
    (second stream) -> epilogue; every step bit-identical to the oracle."""
    import torch

    H, I, E, K, Id = 2816, 704, 128, 8, 2112
    wtype = 2
    h = (synth.normal(60 + T, T * H) * 1.5).reshape(T, H)
    n_ffn, n_pre2, n_gis, p1, p2, p = [norm_weight(synth, 61 + i, H) for i in range(6)]
    W = synth.normal(70, E * H, 0.02).reshape(E, H)
    gu, dn = synth.expert_weights(71, wtype, H, I, E)
    dgu, ddn = synth.expert_weights(72, wtype, H, Id, 1)
    dscale = (1.0 + synth.normal(73, E, 0.05)).astype(np.float32)
    out_scale = 0.5

    _, xs, xm, rx = oracle.ffn_prologue(h, None, None, n_ffn, n_pre2, n_gis)
    _, ids, probs = oracle.router(W, rx, H, E, K, T)
    moe_raw = oracle.experts(wtype, gu, dn, ids, probs, dscale, xm, H, I, E, K, T, n_threads=8)
    mlp_raw = oracle.experts(wtype, dgu, ddn, np.zeros((T, 1), np.int32), np.ones((T, 1), np.float32), None, xs, H,
                             Id, 1, 1, T, n_threads=8)
    want = oracle.ffn_epilogue(h, mlp_raw, moe_raw, p1, p2, p, out_scale)

    g_gu, g_dn = moe.prepare_weights(wtype, dev(gu, cuda), dev(dn, cuda))
    g_dgu, g_ddn = moe.prepare_weights(wtype, dev(dgu, cuda), dev(ddn, cuda))
    wt = wtype | moe.MRML_PACKED
    d_h = dev(h, cuda)
    d_xs, d_xm, d_rx = (torch.empty((T, H), device=cuda) for _ in range(3))
    logits = torch.empty((T, E), device=cuda)
    d_ids = torch.empty((T, K), dtype=torch.int32, device=cuda)
    d_probs = torch.empty((T, K), device=cuda)
    d_moe, d_mlp = torch.empty((T, H), device=cuda), torch.empty((T, H), device=cuda)
    ws = moe.new_workspace(H, I, E, K, T, cuda)
    wsd = moe.new_dense_ffn_workspace(H, Id, T, cuda)
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    moe.ffn_prologue(d_h, None, None, dev(n_ffn, cuda), dev(n_pre2, cuda), dev(n_gis, cuda), None, d_xs, d_xm, d_rx,
                     H, T)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        moe.dense_ffn(wt, g_dgu, g_ddn, d_xs, d_mlp, H, Id, T, wsd, stream=side)
    moe.forward(wt, dev(W, cuda), d_rx, d_xm, g_gu, g_dn, dev(dscale, cuda), logits, d_ids, d_probs, d_moe, H, I, E,
                K, T, ws)
    main.wait_stream(side)
    moe.ffn_epilogue(d_h, d_mlp, d_moe, dev(p1, cuda), dev(p2, cuda), dev(p, cuda), d_h, out_scale, H, T)
    torch.cuda.synchronize()
    assert np.array_equal(d_ids.cpu().numpy(), ids)
    assert_exact(d_moe.cpu().numpy(), moe_raw)
    assert_exact(d_mlp.cpu().numpy(), mlp_raw)
    assert_exact(d_h.cpu().numpy(), want)


@pytest.mark.parametrize("T,with_dense", [(1, True), (8, True), (32, False)])
def test_ffn_block_graph_replays_bit_exact(cuda, moe, oracle, synth, T, with_dense):
    """The whole FFN block (mrml_moe_ffn_block) captured once as a CUDA graph
    (FfnBlockGraph, the reference's capture_layer_ffn_graph) and replayed on
    two decode steps of fresh hidden states: every replay equals the oracle's
    CPU block (model.rs:1719-2196) bit for bit."""
    import torch

    H, I, E, K, Id = 2816, 704, 128, 8, 2112
    wtype = 2
    norms = [norm_weight(synth, 400 + i, H) for i in range(7)]
    W = synth.normal(410, E * H, 0.02).reshape(E, H)
    gu, dn = synth.expert_weights(411, wtype, H, I, E)
    dscale = (1.0 + synth.normal(412, E, 0.05)).astype(np.float32)
    g_gu, g_dn = moe.prepare_weights(wtype, dev(gu, cuda), dev(dn, cuda))
    if with_dense:
        dgu, ddn = synth.expert_weights(413, wtype, H, Id, 1)
        g_dgu, g_ddn = moe.prepare_weights(wtype, dev(dgu, cuda), dev(ddn, cuda))
    else:
        g_dgu = g_ddn = None
    layer_scale = 0.625
    hidden = torch.empty((T, H), device=cuda)
    attn = torch.empty((T, H), device=cuda)
    d_norms = [dev(n, cuda) for n in norms]
    wt = wtype | moe.MRML_PACKED
    G = moe.FfnBlockGraph(wt, wt, hidden, attn, d_norms, layer_scale, dev(W, cuda), g_gu, g_dn, dev(dscale, cuda),
                          g_dgu, g_ddn, H, I, Id if with_dense else 0, E, K, T)
    for step in range(2):
        h = (synth.normal(420 + 2 * step + T, T * H) * 1.5).reshape(T, H)
        a = (synth.normal(421 + 2 * step + T, T * H) * 0.5).reshape(T, H)
        hidden.copy_(dev(h, cuda))
        attn.copy_(dev(a, cuda))
        G.replay()
        torch.cuda.synchronize()
        st, _ = moe.device_status(G.ws)
        assert st == 0
        res, xs, xm, rx = oracle.ffn_prologue(h, a, *norms[:4])
        _, ids, probs = oracle.router(W, rx, H, E, K, T)
        moe_raw = oracle.experts(wtype, gu, dn, ids, probs, dscale, xm, H, I, E, K, T, n_threads=8)
        mlp_raw = (oracle.experts(wtype, dgu, ddn, np.zeros((T, 1), np.int32), np.ones((T, 1), np.float32), None,
                                  xs, H, Id, 1, 1, T, n_threads=8) if with_dense else None)
        want = oracle.ffn_epilogue(res, mlp_raw, moe_raw, *norms[4:], layer_scale)
        assert_exact(hidden.cpu().numpy(), want)
