"""ctypes binding of oracle/libmrml_oracle.so — TEST INFRASTRUCTURE ONLY.

The oracle is the CPU restatement of the reference's MoE path (see
mrml_oracle.h).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use it, and only as the checker or the timed CPU baseline.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmrml_oracle.so")
Q4_0, Q8_0 = 2, 8

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        vp, i, sz, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float
        L.oracle_f16_to_f32.restype = f
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [f]
        for n in ("oracle_quantize_q8_0", "oracle_quantize_q4_0"):
            getattr(L, n).argtypes = [vp, sz, vp]
        for n in ("oracle_dequantize_q4_0", "oracle_dequantize_q8_0"):
            getattr(L, n).argtypes = [vp, sz, vp]
        for n in ("oracle_vec_dot_q4_0_q8_0", "oracle_vec_dot_q8_0_q8_0"):
            getattr(L, n).restype = f
            getattr(L, n).argtypes = [vp, vp, i]
        L.oracle_mat_vec_q8.argtypes = [i, vp, vp, vp, i, i]
        L.oracle_mat_vec_f32.argtypes = [i, vp, vp, vp, i, i]
        L.oracle_gelu_approx.restype = f
        L.oracle_gelu_approx.argtypes = [f]
        L.oracle_geglu.argtypes = [vp, vp, vp, i]
        L.oracle_rms_norm.argtypes = [vp, vp, f, vp, i]
        L.oracle_ffn_prologue.argtypes = [vp] * 10 + [i, i, f]
        L.oracle_ffn_epilogue.argtypes = [vp, vp, vp, vp, vp, vp, f, vp, i, i, f]
        L.oracle_moe_router.argtypes = [vp, vp, vp, vp, vp, i, i, i, i]
        L.oracle_moe_route_from_logits.argtypes = [vp, vp, vp, i, i, i]
        L.oracle_moe_experts.argtypes = [i, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, i]
        L.oracle_moe_expert_trace.argtypes = [i, vp, vp, i, vp, i, i, vp, vp, vp, vp]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def quantize(x, wtype):
    x = _c(x, np.float32)
    n = x.size
    bb = 18 if wtype == Q4_0 else 34
    out = np.zeros(n // 32 * bb, np.uint8)
    fn = lib().oracle_quantize_q4_0 if wtype == Q4_0 else lib().oracle_quantize_q8_0
    fn(_p(x), n, _p(out))
    return out


def dequantize(data, wtype):
    data = _c(data, np.uint8)
    bb = 18 if wtype == Q4_0 else 34
    nb = data.size // bb
    out = np.zeros(nb * 32, np.float32)
    fn = lib().oracle_dequantize_q4_0 if wtype == Q4_0 else lib().oracle_dequantize_q8_0
    fn(_p(data), nb, _p(out))
    return out


def vec_dot(w, a, n, wtype):
    fn = lib().oracle_vec_dot_q4_0_q8_0 if wtype == Q4_0 else lib().oracle_vec_dot_q8_0_q8_0
    return fn(_p(_c(w, np.uint8)), _p(_c(a, np.uint8)), n)


def mat_vec_q8(wtype, w, x_q8, n_rows, n_cols):
    y = np.zeros(n_rows, np.float32)
    lib().oracle_mat_vec_q8(wtype, _p(_c(w, np.uint8)), _p(_c(x_q8, np.uint8)), _p(y), n_rows, n_cols)
    return y


def mat_vec_f32(wtype, w, x, n_rows, n_cols):
    y = np.zeros(n_rows, np.float32)
    lib().oracle_mat_vec_f32(wtype, _p(_c(w, np.uint8)), _p(_c(x, np.float32)), _p(y), n_rows, n_cols)
    return y


def rms_norm(x, weight, eps):
    """Row-wise over a [T, H] array (ops.rs:24-49 per row)."""
    x = _c(x, np.float32)
    T, H = x.shape
    out = np.zeros_like(x)
    w = None if weight is None else _c(weight, np.float32)
    for t in range(T):
        lib().oracle_rms_norm(_p(x[t]), None if w is None else _p(w), eps, _p(out[t]), H)
    return out


def ffn_prologue(hidden, attn, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale, eps=1e-6):
    """(attn_res, x_shared, x_moe, router_x) of model.rs:1719-1784 for [T, H]
    rows; attn None takes hidden as the residual."""
    hidden = _c(hidden, np.float32)
    T, H = hidden.shape
    a = None if attn is None else _c(attn, np.float32)
    outs = [np.zeros_like(hidden) for _ in range(4)]
    ws = [None if w is None else _c(w, np.float32) for w in (post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale)]
    lib().oracle_ffn_prologue(_p(hidden), None if a is None else _p(a), *[None if w is None else _p(w) for w in ws],
                              *[_p(o) for o in outs], H, T, ctypes.c_float(eps))
    return tuple(outs)


def ffn_epilogue(attn_res, mlp_raw, moe_raw, post1, post2, post, out_scale, eps=1e-6):
    """hidden of model.rs:2176-2196 for [T, H] rows (mlp_raw None = zeros)."""
    attn_res, moe_raw = _c(attn_res, np.float32), _c(moe_raw, np.float32)
    T, H = attn_res.shape
    mlp = None if mlp_raw is None else _c(mlp_raw, np.float32)
    ws = [None if w is None else _c(w, np.float32) for w in (post1, post2, post)]
    out = np.zeros_like(attn_res)
    lib().oracle_ffn_epilogue(_p(attn_res), None if mlp is None else _p(mlp), _p(moe_raw),
                              *[None if w is None else _p(w) for w in ws], ctypes.c_float(out_scale), _p(out), H, T,
                              ctypes.c_float(eps))
    return out


def geglu(gate, up):
    gate, up = _c(gate, np.float32), _c(up, np.float32)
    out = np.zeros_like(gate)
    lib().oracle_geglu(_p(gate), _p(up), _p(out), gate.size)
    return out


def router(W, x, H, E, K, T):
    W, x = _c(W, np.float32), _c(x, np.float32)
    logits = np.zeros((T, E), np.float32)
    ids = np.zeros((T, K), np.int32)
    probs = np.zeros((T, K), np.float32)
    lib().oracle_moe_router(_p(W), _p(x), _p(logits), _p(ids), _p(probs), H, E, K, T)
    return logits, ids, probs


def route_from_logits(logits, E, K, T):
    logits = _c(logits, np.float32)
    ids = np.zeros((T, K), np.int32)
    probs = np.zeros((T, K), np.float32)
    lib().oracle_moe_route_from_logits(_p(logits), _p(ids), _p(probs), E, K, T)
    return ids, probs


def experts(wtype, gate_up, down, ids, probs, down_scale, x, H, I, E, K, T, n_threads=1):
    out = np.zeros((T, H), np.float32)
    lib().oracle_moe_experts(wtype, _p(_c(gate_up, np.uint8)), _p(_c(down, np.uint8)), _p(_c(ids, np.int32)),
                             _p(_c(probs, np.float32)),
                             None if down_scale is None else _p(_c(down_scale, np.float32)),
                             _p(_c(x, np.float32)), _p(out), H, I, E, K, T, n_threads)
    return out


def expert_trace(wtype, gate_up, down, expert, x, H, I):
    gate = np.zeros(I, np.float32)
    up = np.zeros(I, np.float32)
    act = np.zeros(I, np.float32)
    dn = np.zeros(H, np.float32)
    lib().oracle_moe_expert_trace(wtype, _p(_c(gate_up, np.uint8)), _p(_c(down, np.uint8)), expert,
                                  _p(_c(x, np.float32)), H, I, _p(gate), _p(up), _p(act), _p(dn))
    return gate, up, act, dn
