"""Host-side mirror of the reference's MoE operator surface over the C ABI.

The reference host is Rust (crates/mrml-tensor/src/cuda.rs); its MoE calls
are methods of `CudaDevice`:

    moe_router(weights, input, logits, ids, probs, dim, n_experts)        cuda.rs:2808
    moe_router_batch(weights, input, logits, ids, probs, dim, n_experts, batch)   :2882
    moe_topk_q4_0(gate_up, down, ids, weights, scales, x_in, act, out,
                  dim, exp_ffn_dim, n_active)                             cuda.rs:2772
    moe_topk_batch_q4_0(..., batch)                                       cuda.rs:2840

`MoeDevice` below keeps those names, argument meanings and size assertions
(the reference asserts buffer lengths and panics on a failed launch; here a
failed assertion raises AssertionError and a failed launch raises MoeError).
Tensors are torch CUDA tensors, used only as device memory; every call goes
through libmrml_moe_b200.so with the tensors' raw pointers.  There is no CPU
fallback: without the library or an sm_100 GPU every call raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmrml_moe_b200.so")

MRML_OK = 0
MRML_ERR_INVALID_ARGUMENT = -1
MRML_Q4_0 = 2
MRML_Q8_0 = 8
MRML_PACKED = 0x100

# Every symbol include/mrml_moe.h declares, with its ctypes signature.
_c = ctypes
_vp, _i, _sz, _f = _c.c_void_p, _c.c_int, _c.c_size_t, _c.c_float
SIGNATURES = {
    "mrml_moe_version": (_i, []),
    "mrml_moe_status_string": (_c.c_char_p, [_i]),
    "mrml_moe_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "mrml_moe_workspace_init": (_i, [_vp, _sz, _vp]),
    "mrml_moe_router": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "mrml_moe_route_from_logits": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "mrml_moe_router_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "mrml_moe_router_logit_bounds": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "mrml_moe_router_noalloc_status": (_i, [_vp]),
    "mrml_moe_experts": (
        _i,
        [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp],
    ),
    "mrml_moe_forward": (
        _i,
        [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp],
    ),
    "mrml_moe_experts_shard": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _sz,
                                    _vp]),
    "mrml_moe_ep_slab_bytes": (_sz, [_i, _i, _i, _i]),
    "mrml_moe_ep_slab_alloc": (_i, [_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "mrml_moe_ep_slab_free": (_i, [_vp]),
    "mrml_moe_ipc_get_handle": (_i, [_vp, _vp]),
    "mrml_moe_ipc_open_handle": (_i, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "mrml_moe_ipc_close_handle": (_i, [_vp]),
    "mrml_moe_ep_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "mrml_moe_ep_dispatch": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "mrml_moe_ep_experts": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "mrml_moe_ep_combine": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "mrml_moe_combine": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "mrml_moe_geglu": (_i, [_vp, _vp, _vp, _sz, _vp]),
    "mrml_moe_rms_norm": (_i, [_vp, _vp, _vp, _i, _i, _f, _vp]),
    "mrml_moe_quantize_q8_0": (_i, [_vp, _vp, _sz, _vp]),
    "mrml_moe_quantize_q4_0": (_i, [_vp, _vp, _sz, _vp]),
    "mrml_moe_device_status": (_i, [_vp, _vp, _c.POINTER(_c.c_int)]),
    "mrml_moe_profile_events": (_i, [_c.POINTER(_vp), _i]),
    "mrml_moe_set_option": (_i, [_i, _i]),
    "mrml_moe_weights_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "mrml_moe_prepare_weights": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "mrml_moe_ffn_prologue": (_i, [_vp] * 10 + [_i, _i, _vp]),
    "mrml_moe_ffn_epilogue": (_i, [_vp] * 7 + [_f, _i, _i, _vp]),
    "mrml_moe_dense_ffn_workspace_bytes": (_sz, [_i, _i, _i]),
    "mrml_moe_ffn_block_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "mrml_moe_ffn_block": (_i, [_i, _i] + [_vp] * 9 + [_f] + [_vp] * 6 + [_i] * 6 + [_vp, _sz, _vp]),
    "mrml_moe_dense_ffn": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "mrml_moe_gguf_open": (_i, [_c.c_char_p, _c.POINTER(_vp)]),
    "mrml_moe_gguf_close": (_i, [_vp]),
    "mrml_moe_gguf_version": (_i, [_vp]),
    "mrml_moe_gguf_tensor_count": (_i, [_vp]),
    "mrml_moe_gguf_tensor_name": (_c.c_char_p, [_vp, _i]),
    "mrml_moe_gguf_tensor": (_i, [_vp, _c.c_char_p, _c.POINTER(_i), _c.POINTER(_i), _c.POINTER(_c.c_int64),
                                  _c.POINTER(_c.c_uint64), _c.POINTER(_c.c_uint64)]),
    "mrml_moe_gguf_meta_u32": (_i, [_vp, _c.c_char_p, _c.POINTER(_c.c_uint32)]),
    "mrml_moe_gguf_read": (_i, [_vp, _c.c_char_p, _vp, _sz]),
}


class MoeError(RuntimeError):
    """A C-ABI call returned a non-zero mrml_status."""

    def __init__(self, what: str, status: int, text: str):
        super().__init__(f"{what} failed: {text} ({status})")
        self.status = status


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libmrml_moe_b200.so (built in-tree by __graft_entry__.build; the
    environment variable MRML_MOE_LIB names another build of it)."""
    global _lib
    if _lib is None:
        path = os.environ.get("MRML_MOE_LIB", path)
        if not os.path.exists(path):
            raise OSError(f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _check(what: str, status: int) -> None:
    if status != MRML_OK:
        text = load_library().mrml_moe_status_string(status).decode()
        raise MoeError(what, status, text)


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    return stream.cuda_stream or None


def workspace_bytes(H: int, I: int, E: int, K: int, T: int) -> int:
    return int(load_library().mrml_moe_workspace_bytes(H, I, E, K, T))


def new_workspace(H: int, I: int, E: int, K: int, T: int, device=None):
    """A zero-initialised, 256-byte aligned device workspace (torch uint8)."""
    import torch

    n = max(256, workspace_bytes(H, I, E, K, T))
    ws = torch.zeros(n, dtype=torch.uint8, device=device or "cuda")
    assert ws.data_ptr() % 256 == 0
    return ws


def router(W, x, logits, ids, probs, H, E, K, T, ws, stream=None):
    lib = load_library()
    _check(
        "mrml_moe_router",
        lib.mrml_moe_router(_ptr(W), _ptr(x), _ptr(logits), _ptr(ids), _ptr(probs), H, E, K, T, _ptr(ws),
                            ws.numel(), _stream_ptr(stream)),
    )


def router_logit_bounds(W, x, lo, hi, H, E, T, stream=None):
    """Intervals [lo, hi] ([T][E]) that contain the router's exact logits."""
    _check("mrml_moe_router_logit_bounds",
           load_library().mrml_moe_router_logit_bounds(_ptr(W), _ptr(x), _ptr(lo), _ptr(hi), H, E, T,
                                                       _stream_ptr(stream)))


def router_noalloc(W, x, logits, ids, probs, H, E, K, T, stream=None):
    """The router without a workspace (scratch kept inside the library); for
    callers that cannot allocate device memory.  T * E must be <= 65536."""
    lib = load_library()
    _check(
        "mrml_moe_router_noalloc",
        lib.mrml_moe_router_noalloc(_ptr(W), _ptr(x), _ptr(logits), _ptr(ids), _ptr(probs), H, E, K, T,
                                    _stream_ptr(stream)),
    )


def route_from_logits(logits, ids, probs, E, K, T, stream=None):
    lib = load_library()
    _check(
        "mrml_moe_route_from_logits",
        lib.mrml_moe_route_from_logits(_ptr(logits), _ptr(ids), _ptr(probs), E, K, T, _stream_ptr(stream)),
    )


def experts(wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, K, T, ws, stream=None):
    lib = load_library()
    _check(
        "mrml_moe_experts",
        lib.mrml_moe_experts(wtype, _ptr(gate_up), _ptr(down), _ptr(ids), _ptr(probs), _ptr(down_scale), _ptr(x),
                             _ptr(out), H, I, E, K, T, _ptr(ws), ws.numel(), _stream_ptr(stream)),
    )


def forward(wtype, router_w, router_x, x, gate_up, down, down_scale, logits, ids, probs, out, H, I, E, K, T, ws,
            stream=None):
    lib = load_library()
    _check(
        "mrml_moe_forward",
        lib.mrml_moe_forward(wtype, _ptr(router_w), _ptr(router_x), _ptr(x), _ptr(gate_up), _ptr(down),
                             _ptr(down_scale), _ptr(logits), _ptr(ids), _ptr(probs), _ptr(out), H, I, E, K, T,
                             _ptr(ws), ws.numel(), _stream_ptr(stream)),
    )


def experts_shard(wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, e_first, e_count, K, T, ws,
                  stream=None):
    lib = load_library()
    _check(
        "mrml_moe_experts_shard",
        lib.mrml_moe_experts_shard(wtype, _ptr(gate_up), _ptr(down), _ptr(ids), _ptr(probs), _ptr(down_scale), _ptr(x),
                                   _ptr(out), H, I, E, e_first, e_count, K, T, _ptr(ws), ws.numel(),
                                   _stream_ptr(stream)),
    )


def ep_slab_alloc(N: int, T: int, H: int, K: int) -> int:
    """Allocates (set-up time) this rank's expert-parallel exchange slab."""
    lib = load_library()
    nbytes = lib.mrml_moe_ep_slab_bytes(N, T, H, K)
    if nbytes == 0:
        raise MoeError("mrml_moe_ep_slab_bytes", MRML_ERR_INVALID_ARGUMENT, "invalid argument")
    p = ctypes.c_void_p()
    _check("mrml_moe_ep_slab_alloc", lib.mrml_moe_ep_slab_alloc(nbytes, ctypes.byref(p)))
    return p.value


def ep_slab_free(ptr: int) -> None:
    _check("mrml_moe_ep_slab_free", load_library().mrml_moe_ep_slab_free(ptr))


def ipc_get_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    _check("mrml_moe_ipc_get_handle", load_library().mrml_moe_ipc_get_handle(ptr, buf))
    return bytes(buf.raw)


def ipc_open_handle(handle: bytes) -> int:
    p = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(handle, 64)
    _check("mrml_moe_ipc_open_handle", load_library().mrml_moe_ipc_open_handle(buf, ctypes.byref(p)))
    return p.value


def ipc_close_handle(ptr: int) -> None:
    _check("mrml_moe_ipc_close_handle", load_library().mrml_moe_ipc_close_handle(ptr))


def new_ep_workspace(N, T, H, I, E, K, device=None):
    """A zeroed workspace for mrml_moe_ep_experts / mrml_moe_ep_combine."""
    import torch

    n = load_library().mrml_moe_ep_workspace_bytes(N, T, H, I, E, K)
    if n == 0:
        raise MoeError("mrml_moe_ep_workspace_bytes", MRML_ERR_INVALID_ARGUMENT, "invalid argument")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def ep_dispatch(slabs, rank, N, T, H, E, K, x, ids, probs, stream=None):
    lib = load_library()
    _check("mrml_moe_ep_dispatch",
           lib.mrml_moe_ep_dispatch(_ptr(slabs), rank, N, T, H, E, K, _ptr(x), _ptr(ids), _ptr(probs),
                                    _stream_ptr(stream)))


def ep_experts(wtype, gate_up, down, down_scale, slabs, rank, N, T, H, I, E, K, ws, stream=None):
    lib = load_library()
    _check("mrml_moe_ep_experts",
           lib.mrml_moe_ep_experts(wtype, _ptr(gate_up), _ptr(down), _ptr(down_scale), _ptr(slabs), rank, N, T, H, I,
                                   E, K, _ptr(ws), ws.numel(), _stream_ptr(stream)))


def ep_combine(slabs, rank, N, T, H, E, K, ids, probs, out, ws, stream=None):
    lib = load_library()
    _check("mrml_moe_ep_combine",
           lib.mrml_moe_ep_combine(_ptr(slabs), rank, N, T, H, E, K, _ptr(ids), _ptr(probs), _ptr(out), _ptr(ws),
                                   _stream_ptr(stream)))


def set_exchange_spin_limit(limit: int) -> None:
    """Poll limit of the exchange's bounded waits (0 = the default)."""
    _check("mrml_moe_set_option", load_library().mrml_moe_set_option(4, limit))


def combine(ydown, pos, ids, probs, down_scale, out, H, K, T, stream=None):
    lib = load_library()
    _check(
        "mrml_moe_combine",
        lib.mrml_moe_combine(_ptr(ydown), _ptr(pos), _ptr(ids), _ptr(probs), _ptr(down_scale), _ptr(out), H, K, T,
                             _stream_ptr(stream)),
    )


def ffn_prologue(hidden, attn, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale, attn_res, shared, moe_in,
                 router_in, dim, batch, stream=None):
    """mrml_moe_ffn_prologue (the reference's prepare_ffn_batch argument
    order); None for an absent input or output."""
    _check("mrml_moe_ffn_prologue",
           load_library().mrml_moe_ffn_prologue(*[_ptr(a) for a in (hidden, attn, post_attn_norm, ffn_norm,
                                                                    pre_ffw_norm_2, router_scale, attn_res, shared,
                                                                    moe_in, router_in)], dim, batch,
                                                _stream_ptr(stream)))


def ffn_epilogue(attn_res, dense, moe_out, post1, post2, post, output, layer_scale, dim, batch, stream=None):
    """mrml_moe_ffn_epilogue (the reference's finish_ffn_batch order)."""
    _check("mrml_moe_ffn_epilogue",
           load_library().mrml_moe_ffn_epilogue(*[_ptr(a) for a in (attn_res, dense, moe_out, post1, post2, post,
                                                                    output)], float(layer_scale), dim, batch,
                                                _stream_ptr(stream)))


def new_dense_ffn_workspace(H, I, T, device=None):
    import torch

    n = load_library().mrml_moe_dense_ffn_workspace_bytes(H, I, T)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def dense_ffn(wtype, gate_up, down, x, out, H, I, T, ws, stream=None):
    _check("mrml_moe_dense_ffn",
           load_library().mrml_moe_dense_ffn(wtype, _ptr(gate_up), _ptr(down), _ptr(x), _ptr(out), H, I, T, _ptr(ws),
                                             ws.numel(), _stream_ptr(stream)))


def new_ffn_block_workspace(H, I, I_dense, E, K, T, device=None):
    import torch

    n = load_library().mrml_moe_ffn_block_workspace_bytes(H, I, I_dense, E, K, T)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def ffn_block(wtype, dense_wtype, hidden, attn, norms, layer_scale, router_w, gate_up, down, down_scale,
              dense_gate_up, dense_down, H, I, I_dense, E, K, T, ws, stream=None):
    """mrml_moe_ffn_block; norms = (post_attn_norm, ffn_norm, pre_ffw_norm_2,
    router_scale, post_ffw_norm_1, post_ffw_norm_2, post_ffw_norm), None for 1."""
    _check("mrml_moe_ffn_block",
           load_library().mrml_moe_ffn_block(wtype, dense_wtype, _ptr(hidden), _ptr(attn), *[_ptr(n) for n in norms],
                                             float(layer_scale), _ptr(router_w), _ptr(gate_up), _ptr(down),
                                             _ptr(down_scale), _ptr(dense_gate_up), _ptr(dense_down), H, I, I_dense,
                                             E, K, T, _ptr(ws), ws.numel(), _stream_ptr(stream)))


class FfnBlockGraph:
    """A layer's FFN block captured once as a CUDA graph and replayed per
    decode step on the device-resident hidden state (the reference's
    capture_layer_ffn_graph, model.rs:295-381, with the block's prepare and
    finish steps inside).  `hidden` and `attn` are the static input buffers:
    write the step's values into them, then replay(); hidden holds the block's
    output afterwards."""

    def __init__(self, wtype, dense_wtype, hidden, attn, norms, layer_scale, router_w, gate_up, down, down_scale,
                 dense_gate_up, dense_down, H, I, I_dense, E, K, T):
        import torch

        self.args = (wtype, dense_wtype, hidden, attn, tuple(norms), layer_scale, router_w, gate_up, down, down_scale,
                     dense_gate_up, dense_down, H, I, I_dense, E, K, T)
        self.ws = new_ffn_block_workspace(H, I, I_dense, E, K, T, hidden.device)
        self.stream = torch.cuda.Stream(hidden.device)
        self.graph = torch.cuda.CUDAGraph()
        self.stream.wait_stream(torch.cuda.current_stream(hidden.device))
        with torch.cuda.graph(self.graph, stream=self.stream):
            ffn_block(*self.args, self.ws, stream=self.stream)

    def replay(self):
        self.graph.replay()


def rms_norm(x, weight, out, dim, batch, eps, stream=None):
    lib = load_library()
    _check("mrml_moe_rms_norm",
           lib.mrml_moe_rms_norm(_ptr(x), _ptr(weight), _ptr(out), dim, batch, eps, _stream_ptr(stream)))


def geglu(gate, up, out, stream=None):
    lib = load_library()
    _check("mrml_moe_geglu", lib.mrml_moe_geglu(_ptr(gate), _ptr(up), _ptr(out), gate.numel(), _stream_ptr(stream)))


def quantize(wtype, src, dst, stream=None):
    lib = load_library()
    fn = lib.mrml_moe_quantize_q4_0 if wtype == MRML_Q4_0 else lib.mrml_moe_quantize_q8_0
    _check("mrml_moe_quantize", fn(_ptr(src), _ptr(dst), src.numel(), _stream_ptr(stream)))


OPTION_EXPERT_PATH = 1
PATH_AUTO, PATH_GEMV, PATH_TENSOR, PATH_GENERAL = 0, 1, 2, 3


def prepare_weights(wtype, gate_up, down, stream=None):
    """Repacks one layer's GGUF expert slabs into the decode kernel's layout
    (mrml_moe_prepare_weights); returns (gate_up_packed, down_packed), device
    tensors of the same sizes, to be passed with wtype | MRML_PACKED."""
    import torch

    lib = load_library()
    gp = torch.empty_like(gate_up)
    dp = torch.empty_like(down)
    _check("mrml_moe_prepare_weights",
           lib.mrml_moe_prepare_weights(wtype, _ptr(gate_up), _ptr(down), _ptr(gp), _ptr(dp), *_prep_shape(
               wtype, gate_up, down), _stream_ptr(stream)))
    return gp, dp


def _prep_shape(wtype, gate_up, down):
    """(H, I, E) of GGUF slabs shaped [E][2I][H/32*bb] and [E][H][I/32*bb]."""
    bb = 18 if (wtype & 0xff) == MRML_Q4_0 else 34
    E, two_i, row = gate_up.shape
    return row // bb * 32, two_i // 2, E


def set_expert_path(path: int) -> None:
    """0 automatic, 1 pipelined CUDA-core kernels, 2 tcgen05 tensor cores,
    3 general CUDA-core kernels (process-wide)."""
    _check("mrml_moe_set_option", load_library().mrml_moe_set_option(OPTION_EXPERT_PATH, path))


OPTION_SPECULATIVE_ROUTING = 5


def set_speculative_routing(on: bool) -> None:
    """Speculative routing of batches up to 32 tokens in forward (default off;
    results are identical either way)."""
    _check("mrml_moe_set_option", load_library().mrml_moe_set_option(OPTION_SPECULATIVE_ROUTING, 1 if on else 0))


def device_status(ws, stream=None):
    """(status, 0); synchronises the stream.  The second value is the
    header's recomputed-token count, always 0 (the router is exact)."""
    lib = load_library()
    rec = ctypes.c_int(0)
    st = lib.mrml_moe_device_status(_ptr(ws), _stream_ptr(stream), ctypes.byref(rec))
    return st, rec.value


class GgufFile:
    """A GGUF file's tensor table through mrml_moe_gguf_* (the reference's
    reader, crates/mrml-tensor/src/gguf.rs:80-181).  Host only."""

    def __init__(self, path: str):
        lib = load_library()
        h = ctypes.c_void_p()
        _check("mrml_moe_gguf_open", lib.mrml_moe_gguf_open(os.fsencode(path), ctypes.byref(h)))
        self._h = h
        self.version = lib.mrml_moe_gguf_version(h)

    def close(self):
        if self._h:
            load_library().mrml_moe_gguf_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def names(self):
        lib = load_library()
        return [lib.mrml_moe_gguf_tensor_name(self._h, i).decode() for i in range(lib.mrml_moe_gguf_tensor_count(self._h))]

    def tensor(self, name: str):
        """{type, dims (innermost first), offset (absolute), nbytes} or None."""
        t, nd = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        st = load_library().mrml_moe_gguf_tensor(self._h, name.encode(), ctypes.byref(t), ctypes.byref(nd), dims,
                                                 ctypes.byref(off), ctypes.byref(nb))
        if st == -8:
            return None
        _check("mrml_moe_gguf_tensor", st)
        return {"type": t.value, "dims": tuple(dims[:nd.value]), "offset": off.value, "nbytes": nb.value}

    def meta_u32(self, key: str):
        v = ctypes.c_uint32()
        st = load_library().mrml_moe_gguf_meta_u32(self._h, key.encode(), ctypes.byref(v))
        if st == -8:
            return None
        _check("mrml_moe_gguf_meta_u32", st)
        return v.value

    def read(self, name: str):
        """The tensor's bytes (numpy uint8)."""
        import numpy as np

        info = self.tensor(name)
        if info is None:
            raise MoeError("mrml_moe_gguf_read", -8, f"no tensor {name}")
        buf = np.empty(info["nbytes"], np.uint8)
        _check("mrml_moe_gguf_read", load_library().mrml_moe_gguf_read(self._h, name.encode(),
                                                                        buf.ctypes.data_as(ctypes.c_void_p),
                                                                        buf.size))
        return buf


def load_moe_layer(gguf, layer: int, device, packed: bool = False, stream=None) -> dict:
    """One MoE layer's tensors as the reference's loader takes them
    (model.rs:630-755): the router `blk.{l}.ffn_gate_inp.weight` [E][H] f32,
    its optional `.scale` [H], the expert slabs `blk.{l}.ffn_gate_up_exps.weight`
    ([E][2I][H/32] blocks) and `ffn_down_exps.weight` ([E][H][I/32] blocks),
    uploaded unchanged, and the optional `ffn_down_exps.scale` [E].  With
    packed=True the slabs are repacked on the device (mrml_moe_prepare_weights)
    and `wtype` carries MRML_PACKED.  `gguf` is a path or an open GgufFile."""
    import numpy as np
    import torch

    own = isinstance(gguf, (str, bytes, os.PathLike))
    g = GgufFile(gguf) if own else gguf
    try:
        pre = f"blk.{layer}."
        gu_i, dn_i = g.tensor(pre + "ffn_gate_up_exps.weight"), g.tensor(pre + "ffn_down_exps.weight")
        if gu_i is None or dn_i is None:
            raise MoeError("load_moe_layer", -8, f"layer {layer} has no expert slabs")
        wtype = gu_i["type"]
        if wtype not in (MRML_Q4_0, MRML_Q8_0) or dn_i["type"] != wtype:
            raise MoeError("load_moe_layer", -2, f"expert weight type {wtype}")
        H, two_i, E = gu_i["dims"][:3]
        I = two_i // 2
        if tuple(dn_i["dims"][:3]) != (I, H, E):
            raise MoeError("load_moe_layer", -1, "gate_up and down slabs disagree")
        bb = 18 if wtype == MRML_Q4_0 else 34

        def dev(a, shape=None, dtype=None):
            t = torch.from_numpy(a if dtype is None else a.view(dtype))
            return (t if shape is None else t.reshape(shape)).to(device)

        out = {"wtype": wtype, "H": H, "I": I, "E": E,
               "gate_up": dev(g.read(pre + "ffn_gate_up_exps.weight"), (E, 2 * I, H // 32 * bb)),
               "down": dev(g.read(pre + "ffn_down_exps.weight"), (E, H, I // 32 * bb))}
        for key, name, shape in (("router_w", "ffn_gate_inp.weight", (E, H)), ("gate_inp_scale", "ffn_gate_inp.scale",
                                                                               (H,)),
                                 ("down_scale", "ffn_down_exps.scale", (E,))):
            info = g.tensor(pre + name)
            out[key] = None if info is None or info["type"] != 0 else dev(g.read(pre + name), shape, np.float32)
        if packed:
            out["gate_up"], out["down"] = prepare_weights(wtype, out["gate_up"], out["down"], stream)
            out["wtype"] = wtype | MRML_PACKED
        return out
    finally:
        if own:
            g.close()


class MoeDevice:
    """The reference's `CudaDevice` MoE methods (cuda.rs:2772-2912) on the
    B200 library.  Holds one workspace, grown on demand; grow it (call
    `reserve`) before capturing a CUDA graph."""

    def __init__(self, device_id: int = 0):
        import torch

        self.device = torch.device("cuda", device_id)
        self._ws = None
        self._ws_shape = None

    def reserve(self, H: int, I: int, E: int, K: int, T: int):
        need = workspace_bytes(H, I, E, K, T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = new_workspace(H, I, E, K, T, self.device)
        return self._ws

    # cuda.rs:2808-2838 (T = 1, K = 8)
    def moe_router(self, d_weights, d_input, d_logits, d_ids, d_probabilities, dim, n_experts, k=8):
        assert d_weights.numel() >= dim * n_experts
        assert d_input.numel() >= dim
        assert d_logits.numel() >= n_experts
        assert d_ids.numel() >= k
        assert d_probabilities.numel() >= k
        ws = self.reserve(32, 32, n_experts, k, 1)
        router(d_weights, d_input, d_logits, d_ids, d_probabilities, dim, n_experts, k, 1, ws)

    # cuda.rs:2882-2912
    def moe_router_batch(self, weights, input, logits, ids, probabilities, dim, n_experts, batch, k=8):
        assert input.numel() == dim * batch
        assert logits.numel() == n_experts * batch
        assert ids.numel() == k * batch
        assert probabilities.numel() == k * batch
        ws = self.reserve(32, 32, n_experts, k, batch)
        router(weights, input, logits, ids, probabilities, dim, n_experts, k, batch, ws)

    # cuda.rs:2772-2806.  `d_act_scratch` is accepted for signature parity;
    # the library uses its own workspace for the GeGLU activations.
    def moe_topk_q4_0(self, d_gate_up_exps, d_down_exps, d_active_exp_ids, d_active_exp_weights,
                      d_down_exps_scale, d_x_in, d_act_scratch, d_out_moe, dim, exp_ffn_dim, n_active,
                      n_experts=None, wtype=MRML_Q4_0):
        E = n_experts or self._infer_experts(d_gate_up_exps, dim, exp_ffn_dim, wtype)
        ws = self.reserve(dim, exp_ffn_dim, E, n_active, 1)
        experts(wtype, d_gate_up_exps, d_down_exps, d_active_exp_ids, d_active_exp_weights, d_down_exps_scale,
                d_x_in, d_out_moe, dim, exp_ffn_dim, E, n_active, 1, ws)

    # cuda.rs:2840-2880
    def moe_topk_batch_q4_0(self, gate_up, down, ids, weights, scales, input, act, output, dim, exp_dim,
                            n_active, batch, n_experts=None, wtype=MRML_Q4_0):
        assert ids.numel() == batch * n_active
        assert weights.numel() == batch * n_active
        assert input.numel() == batch * dim
        assert output.numel() == batch * dim
        E = n_experts or self._infer_experts(gate_up, dim, exp_dim, wtype)
        ws = self.reserve(dim, exp_dim, E, n_active, batch)
        experts(wtype, gate_up, down, ids, weights, scales, input, output, dim, exp_dim, E, n_active, batch, ws)

    # cuda.rs:2914-2947 (batch 1) and 2949-2985
    def prepare_ffn(self, hidden, attn_proj, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale, attn_res,
                    shared_in, moe_in, router_in, dim):
        ffn_prologue(hidden, attn_proj, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale, attn_res, shared_in,
                     moe_in, router_in, dim, 1)

    def prepare_ffn_batch(self, hidden, attn, pan, ffn, pfn, router_scale, attn_res, shared, moe_in, router_in, dim,
                          batch):
        assert hidden.numel() == dim * batch
        assert attn.numel() == dim * batch
        ffn_prologue(hidden, attn, pan, ffn, pfn, router_scale, attn_res, shared, moe_in, router_in, dim, batch)

    # cuda.rs:2987-3016 (batch 1) and 3018-3050
    def finish_ffn(self, attn_res, dense, moe_out, post_ffw_norm_1, post_ffw_norm_2, post_ffw_norm, hidden_out,
                   layer_scale, dim):
        ffn_epilogue(attn_res, dense, moe_out, post_ffw_norm_1, post_ffw_norm_2, post_ffw_norm, hidden_out,
                     layer_scale, dim, 1)

    def finish_ffn_batch(self, attn_res, dense, moe_out, p1, p2, pf, output, scale, dim, batch):
        assert attn_res.numel() == dim * batch
        assert output.numel() == dim * batch
        ffn_epilogue(attn_res, dense, moe_out, p1, p2, pf, output, scale, dim, batch)

    @staticmethod
    def _infer_experts(gate_up, dim, exp_dim, wtype):
        bb = 18 if wtype == MRML_Q4_0 else 34
        per_expert = 2 * exp_dim * (dim // 32) * bb
        assert gate_up.numel() % per_expert == 0, "gate_up size is not a whole number of experts"
        return gate_up.numel() // per_expert
