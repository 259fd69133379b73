"""GGUF tensor-table reader (mrml_moe_gguf_*) and the MoE layer loader.

The files are written here by a small GGUF v3 writer that follows the format
the reference reads (crates/mrml-tensor/src/gguf.rs:80-181): header, typed
metadata (every value type, arrays included), tensor infos, then the data
section aligned to general.alignment.
"""

from __future__ import annotations

import struct

import numpy as np
import pytest

GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, GGUF_STR, GGUF_ARR, GGUF_U64, \
    GGUF_I64, GGUF_F64 = range(13)
_FMT = {GGUF_U8: "<B", GGUF_I8: "<b", GGUF_U16: "<H", GGUF_I16: "<h", GGUF_U32: "<I", GGUF_I32: "<i",
        GGUF_F32: "<f", GGUF_BOOL: "<B", GGUF_U64: "<Q", GGUF_I64: "<q", GGUF_F64: "<d"}
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 30: (1, 2)}


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _val(vt, v):
    if vt == GGUF_STR:
        return _str(v)
    if vt == GGUF_ARR:
        it, items = v
        return struct.pack("<IQ", it, len(items)) + b"".join(_val(it, x) for x in items)
    return struct.pack(_FMT[vt], v)


def write_gguf(path, meta, tensors, alignment=None, version=3):
    """meta: [(key, type, value)]; tensors: [(name, ggml_type, dims innermost
    first, bytes)].  Returns {name: absolute data offset}."""
    meta = list(meta)
    if alignment is not None:
        meta.append(("general.alignment", GGUF_U32, alignment))
    align = alignment or 32
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(meta))
    head += b"".join(_str(k) + struct.pack("<I", t) + _val(t, v) for k, t, v in meta)
    offsets, rel = {}, 0
    infos = b""
    for name, gt, dims, data in tensors:
        rel = -(-rel // align) * align
        infos += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", gt, rel)
        offsets[name] = rel
        rel += len(data)
    head += infos
    data_off = -(-len(head) // align) * align
    blob = bytearray(head + b"\0" * (data_off - len(head)))
    for name, gt, dims, data in tensors:
        start = data_off + offsets[name]
        blob += b"\0" * (start - len(blob))
        blob += bytes(data)
    with open(path, "wb") as f:
        f.write(blob)
    return {n: data_off + o for n, o in offsets.items()}


def moe_layer_tensors(synth, layer, wtype, H, I, E, seed):
    """One layer's MoE tensors in the GGUF shapes the reference loads."""
    gu, dn = synth.expert_weights(seed, wtype, H, I, E)
    W = synth.normal(seed + 1, E * H, 0.02).reshape(E, H)
    dscale = (0.5 + synth.normal(seed + 2, E, 0.1)).astype(np.float32)
    p = f"blk.{layer}."
    return [(p + "ffn_gate_inp.weight", 0, [H, E], W.astype(np.float32).tobytes()),
            (p + "ffn_gate_up_exps.weight", wtype, [H, 2 * I, E], gu.tobytes()),
            (p + "ffn_down_exps.weight", wtype, [I, H, E], dn.tobytes()),
            (p + "ffn_down_exps.scale", 0, [E], dscale.tobytes())], (gu, dn, W, dscale)


META = [("general.architecture", GGUF_STR, "gemma4"), ("gemma4.expert_count", GGUF_U32, 8),
        ("gemma4.expert_used_count", GGUF_I32, 2), ("x.u8", GGUF_U8, 7), ("x.i8", GGUF_I8, -3),
        ("x.u16", GGUF_U16, 513), ("x.i16", GGUF_I16, -2), ("x.f32", GGUF_F32, 1.5), ("x.bool", GGUF_BOOL, 1),
        ("x.u64", GGUF_U64, 1 << 33), ("x.i64", GGUF_I64, -9), ("x.f64", GGUF_F64, 2.25),
        ("x.arr", GGUF_ARR, (GGUF_STR, ["a", "bc"])), ("x.nested", GGUF_ARR, (GGUF_ARR, [(GGUF_I32, [1, 2])]))]


@pytest.mark.parametrize("alignment", [None, 64])
def test_gguf_reader_matches_written_file(tmp_path, moe, synth, alignment):
    tensors, (gu, dn, W, dscale) = moe_layer_tensors(synth, 3, 2, 256, 128, 4, 21)
    tensors.append(("token_embd.weight", 1, [256, 10, 1, 1, 1], np.zeros(2560, np.float16).tobytes()))
    path = str(tmp_path / "m.gguf")
    offs = write_gguf(path, META, tensors, alignment)
    with moe.GgufFile(path) as g:
        assert g.version == 3
        assert g.names() == [t[0] for t in tensors]
        for name, gt, dims, data in tensors:
            info = g.tensor(name)
            assert info["type"] == gt and info["offset"] == offs[name] and info["nbytes"] == len(data)
            assert info["dims"] == tuple(dims[:4])  # a fifth dimension is read and dropped
            assert g.read(name).tobytes() == data
        assert g.tensor("blk.9.ffn_down_exps.weight") is None
        assert g.meta_u32("gemma4.expert_count") == 8 and g.meta_u32("gemma4.expert_used_count") == 2
        assert g.meta_u32("x.u16") == 513 and g.meta_u32("x.u8") == 7
        assert g.meta_u32("x.i8") is None  # as_u32 takes neither i8 nor floats
        assert g.meta_u32("x.f32") is None and g.meta_u32("missing") is None


def test_gguf_reader_rejects_bad_files(tmp_path, moe):
    lib = moe.load_library()
    import ctypes

    h = ctypes.c_void_p()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 64)
    assert lib.mrml_moe_gguf_open(str(bad).encode(), ctypes.byref(h)) == -1
    old = tmp_path / "v1.gguf"
    write_gguf(str(old), [], [], version=1)
    assert lib.mrml_moe_gguf_open(str(old).encode(), ctypes.byref(h)) == -2
    odd = tmp_path / "odd.gguf"
    write_gguf(str(odd), [], [("t", 99, [32], b"\0" * 32)])  # a type the reference does not read
    assert lib.mrml_moe_gguf_open(str(odd).encode(), ctypes.byref(h)) == -2
    cut = tmp_path / "cut.gguf"
    write_gguf(str(cut), META, [])
    cut.write_bytes(cut.read_bytes()[:40])
    assert lib.mrml_moe_gguf_open(str(cut).encode(), ctypes.byref(h)) == -1
    assert lib.mrml_moe_gguf_open(str(tmp_path / "none.gguf").encode(), ctypes.byref(h)) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("packed", [False, True])
def test_loaded_layer_runs_bit_exact(tmp_path, cuda, moe, oracle, synth, packed):
    """A MoE layer written to a GGUF file, loaded back (optionally repacked)
    and run through mrml_moe_forward: bit-identical to the oracle on the
    written tensors."""
    import torch

    H, I, E, K, T, wtype = 256, 128, 8, 2, 5, 2
    tensors, (gu, dn, W, dscale) = moe_layer_tensors(synth, 0, wtype, H, I, E, 31)
    path = str(tmp_path / "layer.gguf")
    write_gguf(path, META, tensors, 64)
    L = moe.load_moe_layer(path, 0, cuda, packed=packed)
    assert (L["H"], L["I"], L["E"]) == (H, I, E) and L["gate_inp_scale"] is None
    x = synth.normal(32, T * H).reshape(T, H)
    d_x = torch.from_numpy(x).to(cuda)
    logits = torch.empty(T, E, device=cuda)
    ids = torch.empty(T, K, dtype=torch.int32, device=cuda)
    probs = torch.empty(T, K, device=cuda)
    out = torch.empty(T, H, device=cuda)
    ws = moe.new_workspace(H, I, E, K, T, cuda)
    moe.forward(L["wtype"], L["router_w"], d_x, d_x, L["gate_up"], L["down"], L["down_scale"], logits, ids, probs, out,
                H, I, E, K, T, ws)
    assert moe.device_status(ws)[0] == 0
    _, r_ids, r_probs = oracle.router(W, x, H, E, K, T)
    ref = oracle.experts(wtype, gu, dn, r_ids, r_probs, dscale, x, H, I, E, K, T)
    assert np.array_equal(ids.cpu().numpy(), r_ids)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
