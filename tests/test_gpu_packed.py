"""Packed expert weights (mrml_moe_prepare_weights).

The packed layout reorders each layer's GGUF expert bytes by MMA fragment
(same bytes, same size).  Checked here:
  * the device repack against a numpy restatement of the layout, byte for
    byte, for Q4_0 and Q8_0;
  * the layer computed from packed weights against the oracle (bit-exact),
    on the decode (dp4a and warp-MMA), half-chain and 16-position forms;
  * argument checks (unsupported shapes, overlapping buffers).
"""

from __future__ import annotations

import numpy as np
import pytest

from test_gpu_parity import Layer, assert_exact, dev_tensor, make_layer_inputs

pytestmark = pytest.mark.gpu


def repack_numpy(raw, wtype, which, H, I, E):
    """The packed layout, restated: records of (16-row tile, block) in MMA
    fragment order; gate_up grouped [E][part][64-row group][K chunk of 8
    blocks][tile 4][block 8], down [E][128-row group][K chunk of kc
    blocks][tile 8][block kc], kc the largest divisor of I/32 up to 12."""
    bb = 18 if wtype == 2 else 34
    rows_part, parts, nb = (I, 2, H // 32) if which == 0 else (H, 1, I // 32)
    blocks = np.asarray(raw, np.uint8).reshape(E, parts, rows_part, nb, bb)
    d16 = blocks[..., :2]
    vals = blocks[..., 2:]
    nw = (bb - 2) // 4
    words = vals.reshape(E, parts, rows_part, nb, nw, 4)
    RB = 16 * bb
    out = np.zeros((E * parts * rows_part * nb // 16, RB), np.uint8)
    r = np.arange(rows_part)
    b = np.arange(nb)
    if which == 0:
        nG, nC = rows_part // 64, nb // 8
        G, j, c, bl = r // 64, (r % 64) // 16, b // 8, b % 8
        rec = (((((np.arange(E)[:, None, None, None] * parts + np.arange(parts)[None, :, None, None]) * nG
                  + G[None, None, :, None]) * nC + c[None, None, None, :]) * 4 + j[None, None, :, None]) * 8
               + bl[None, None, None, :])
    else:
        kc = max(c for c in range(1, min(nb, 12) + 1) if nb % c == 0)
        nG, nC = rows_part // 128, nb // kc
        G, j, c, bl = r // 128, (r % 128) // 16, b // kc, b % kc
        rec = ((((np.arange(E)[:, None, None, None] * nG + G[None, None, :, None]) * nC + c[None, None, None, :]) * 8
                + j[None, None, :, None]) * kc + bl[None, None, None, :])
        rec = np.broadcast_to(rec, (E, parts, rows_part, nb))
    rr = r % 16
    g, h = rr % 8, rr // 8
    flat_rec = rec.reshape(-1)
    gg = np.broadcast_to(g[None, None, :, None], rec.shape).reshape(-1)
    hh = np.broadcast_to(h[None, None, :, None], rec.shape).reshape(-1)
    W = words.reshape(-1, nw, 4)
    D = d16.reshape(-1, 2)
    vb = 256 if wtype == 2 else 512
    for t in range(4):
        if wtype == 2:
            off = 8 * (4 * gg + t) + 4 * hh
            for k in range(4):
                out[flat_rec, off + k] = W[:, t, k]
        else:
            off = 16 * (4 * gg + t) + 4 * hh
            for k in range(4):
                out[flat_rec, off + k] = W[:, t, k]
                out[flat_rec, off + 8 + k] = W[:, 4 + t, k]
    soff = vb + 4 * gg + 2 * hh
    out[flat_rec, soff] = D[:, 0]
    out[flat_rec, soff + 1] = D[:, 1]
    return out.reshape(-1)


@pytest.mark.parametrize("wtype,H,I,E", [(2, 256, 128, 3), (8, 512, 192, 2), (2, 2816, 704, 2)])
def test_repack_matches_layout(cuda, moe, synth, wtype, H, I, E):
    gu, dn = synth.expert_weights(11, wtype, H, I, E)
    gp, dp = moe.prepare_weights(wtype, dev_tensor(gu, cuda), dev_tensor(dn, cuda))
    assert np.array_equal(gp.cpu().numpy().reshape(-1), repack_numpy(gu, wtype, 0, H, I, E))
    assert np.array_equal(dp.cpu().numpy().reshape(-1), repack_numpy(dn, wtype, 1, H, I, E))


class PackedLayer(Layer):
    """A Layer whose expert weights are repacked on the device."""

    def __init__(self, moe, device, wtype, gu, dn, W, H, I, E, K, T, down_scale=None):
        super().__init__(moe, device, wtype, gu, dn, W, H, I, E, K, T, down_scale)
        self.gu, self.dn = moe.prepare_weights(wtype, self.gu, self.dn)
        self.wtype = wtype | moe.MRML_PACKED


PATHS = {"auto": 0, "gemv_dp4a": 1, "gemv_mma": 4}


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("wtype,H,I,E,K,T", [(2, 2816, 704, 32, 8, 1), (2, 2816, 704, 32, 8, 8),
                                              (2, 2816, 704, 32, 8, 64), (8, 1024, 512, 16, 2, 4),
                                              (8, 2816, 704, 16, 8, 9), (2, 1024, 512, 16, 2, 300),
                                              (8, 512, 128, 8, 4, 100)])
def test_packed_layer_bit_exact(cuda, moe, oracle, synth, path, wtype, H, I, E, K, T):
    gu, dn, W, x = make_layer_inputs(synth, wtype, H, I, E, T, seed=H + I + E + T)
    scale = (0.5 + synth.normal(78, E, 0.1)).astype(np.float32)
    L = PackedLayer(moe, cuda, wtype, gu, dn, W, H, I, E, K, T, scale)
    _, r_ids, r_probs = oracle.router(W, x, H, E, K, T)
    moe.set_expert_path(PATHS[path])
    try:
        got = L.experts(x, r_ids, r_probs)
    finally:
        moe.set_expert_path(0)
    ref = oracle.experts(wtype, gu, dn, r_ids, r_probs, scale, x, H, I, E, K, T, 8)
    assert_exact(got, ref)


def test_packed_forward_config2_t64(cuda, moe, oracle, synth):
    """The headline shape through mrml_moe_forward with packed weights."""
    H, I, E, K, T = 2816, 704, 128, 8, 64
    gu, dn = synth.expert_weights_device(2, 2, H, I, E, cuda, moe.quantize)
    gu, dn = gu.cpu().numpy(), dn.cpu().numpy()
    W = synth.normal(33, E * H, 0.02).reshape(E, H)
    x = synth.normal(34 + T, T * H).reshape(T, H)
    L = PackedLayer(moe, cuda, 2, gu, dn, W, H, I, E, K, T)
    ids, probs, out, _ = L.forward(x)
    _, r_ids, r_probs = oracle.router(W, x, H, E, K, T)
    assert np.array_equal(ids, r_ids)
    assert_exact(out, oracle.experts(2, gu, dn, r_ids, r_probs, None, x, H, I, E, K, T, 8))


def test_prepare_weights_rejects_bad_arguments(cuda, moe, synth):
    import torch

    lib = moe.load_library()
    H, I, E = 256, 96, 2  # I not a multiple of 64: no packed layout
    gu = torch.zeros((E, 2 * I, H // 32 * 18), dtype=torch.uint8, device=cuda)
    dn = torch.zeros((E, H, I // 32 * 18), dtype=torch.uint8, device=cuda)
    gp, dp = torch.empty_like(gu), torch.empty_like(dn)  # held, so that the two outputs are distinct buffers
    st = lib.mrml_moe_prepare_weights(2, gu.data_ptr(), dn.data_ptr(), gp.data_ptr(), dp.data_ptr(), H, I, E, None)
    assert st == -2
    H, I = 256, 128
    gu = torch.zeros((E, 2 * I, H // 32 * 18), dtype=torch.uint8, device=cuda)
    dn = torch.zeros((E, H, I // 32 * 18), dtype=torch.uint8, device=cuda)
    # in place (output overlapping the input) is refused
    dp = torch.empty_like(dn)
    st = lib.mrml_moe_prepare_weights(2, gu.data_ptr(), dn.data_ptr(), gu.data_ptr(), dp.data_ptr(), H, I, E, None)
    assert st == -1
    assert lib.mrml_moe_weights_bytes(2, H, I, E, 0) == gu.numel()
    assert lib.mrml_moe_weights_bytes(2, H, I, E, 1) == dn.numel()
