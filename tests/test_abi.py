"""The C-ABI library: it loads, exports every declared symbol, and rejects
bad arguments before touching a GPU (no compute call runs here)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mrml_moe.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mrml_moe_\w+)\s*\(", text)))


def test_header_declares_the_operator_surface():
    names = declared_functions()
    for needed in ("mrml_moe_router", "mrml_moe_experts", "mrml_moe_forward", "mrml_moe_route_from_logits",
                   "mrml_moe_workspace_bytes", "mrml_moe_status_string", "mrml_moe_device_status"):
        assert needed in names


def test_library_exports_every_declared_symbol(moe):
    lib = moe.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in moe.SIGNATURES, f"{name} has no ctypes signature"


def test_library_is_built_for_sm100a():
    # The fatbin's target is recorded in the ELF; check via cuobjdump-free
    # means: the build flags are fixed in build.py.
    import importlib.util

    spec = importlib.util.spec_from_file_location("b", os.path.join(ROOT, "qt_llama.cpp_b200", "build.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    assert "arch=compute_100a,code=sm_100a" in b.NVCC_FLAGS
    assert not any("fast-math" in f or "fast_math" in f for f in b.NVCC_FLAGS)


def test_status_strings(moe):
    lib = moe.load_library()
    assert lib.mrml_moe_status_string(0) == b"ok"
    for code in range(-7, 0):
        assert lib.mrml_moe_status_string(code) != b"unknown status"


def test_workspace_bytes(moe):
    lib = moe.load_library()
    small = lib.mrml_moe_workspace_bytes(1024, 512, 16, 2, 4)
    big = lib.mrml_moe_workspace_bytes(1024, 512, 16, 2, 2048)
    assert small > 0 and small % 256 == 0 and big > small
    assert lib.mrml_moe_workspace_bytes(-1, 512, 16, 2, 4) == 0


def test_invalid_arguments_rejected_without_a_gpu(moe):
    lib = moe.load_library()
    P = ctypes.c_void_p(0x1000)
    # K > E, E over the limit, H not a multiple of 32, unknown weight type.
    assert lib.mrml_moe_router(P, P, P, P, P, 64, 4, 8, 1, P, 1 << 20, None) == -1
    assert lib.mrml_moe_router(P, P, P, P, P, 64, 512, 8, 1, P, 1 << 20, None) == -2
    assert lib.mrml_moe_experts(2, P, P, P, P, None, P, P, 100, 64, 8, 2, 1, P, 1 << 20, None) == -1
    assert lib.mrml_moe_experts(3, P, P, P, P, None, P, P, 64, 64, 8, 2, 1, P, 1 << 20, None) == -2
    # Misaligned weights.
    assert lib.mrml_moe_experts(2, ctypes.c_void_p(0x1001), P, P, P, None, P, P, 64, 64, 8, 2, 1, P, 1 << 20,
                                None) == -1
    # Null pointers with work to do.
    assert lib.mrml_moe_experts(2, None, P, P, P, None, P, P, 64, 64, 8, 2, 1, P, 1 << 20, None) == -1
    assert lib.mrml_moe_quantize_q8_0(P, P, 33, None) == -1
    # Expert shards: the range must lie inside [0, E).
    shard = lib.mrml_moe_experts_shard
    assert shard(2, P, P, P, P, None, P, P, 64, 64, 8, 6, 4, 2, 1, P, 1 << 20, None) == -1
    assert shard(2, P, P, P, P, None, P, P, 64, 64, 8, -1, 4, 2, 1, P, 1 << 20, None) == -1
    assert shard(2, P, P, P, P, None, P, P, 64, 64, 8, 0, 0, 2, 1, P, 1 << 20, None) == -1
    assert shard(2, P, P, P, P, None, P, P, 64, 64, 512, 0, 4, 2, 1, P, 1 << 20, None) == -1
    assert lib.mrml_moe_combine(P, P, P, P, None, P, 64, 65, 1, None) == -1
    assert lib.mrml_moe_rms_norm(P, None, P, 0, 1, ctypes.c_float(1e-6), None) == -1
    assert lib.mrml_moe_rms_norm(ctypes.c_void_p(0x1004), None, P, 64, 1, ctypes.c_float(1e-6), None) == -1
    assert lib.mrml_moe_rms_norm(P, None, P, 1 << 20, 1, ctypes.c_float(1e-6), None) == -2
    # FFN prologue / epilogue and the shared dense MLP.
    N = None
    assert lib.mrml_moe_ffn_prologue(P, P, N, N, N, N, N, N, N, N, 2816, 1, None) == -1  # no output
    assert lib.mrml_moe_ffn_prologue(N, P, N, N, N, N, P, N, N, N, 2816, 1, None) == -1  # no hidden
    assert lib.mrml_moe_ffn_prologue(P, N, N, N, N, N, P, N, N, N, 1 << 20, 1, None) == -2
    assert lib.mrml_moe_ffn_prologue(N, N, N, N, N, N, N, N, N, N, 2816, 0, None) == 0
    assert lib.mrml_moe_ffn_epilogue(P, N, N, N, N, N, P, ctypes.c_float(1), 2816, 1, None) == -1  # no moe
    assert lib.mrml_moe_ffn_epilogue(P, N, P, N, N, N, P, ctypes.c_float(1), 1 << 20, 1, None) == -2
    assert lib.mrml_moe_ffn_block_workspace_bytes(2816, 704, 2112, 128, 8, 64) > 0
    assert lib.mrml_moe_ffn_block_workspace_bytes(2816, 704, -1, 128, 8, 64) == 0
    blk = lib.mrml_moe_ffn_block
    nine = [P] + [None] * 8
    assert blk(2, 2, *nine, ctypes.c_float(1), None, P, P, None, None, None, 2816, 704, 0, 128, 8, 1, P, 1 << 30,
               None) == -1  # no router weights
    assert blk(2, 2, *nine, ctypes.c_float(1), P, P, P, None, None, None, 2816, 704, 2112, 128, 8, 1, P, 1 << 30,
               None) == -1  # a shared MLP without its slabs
    assert blk(2, 2, *nine, ctypes.c_float(1), P, P, P, None, None, None, 2816, 704, 0, 128, 8, 1, P, 16,
               None) == -3
    assert lib.mrml_moe_dense_ffn_workspace_bytes(2816, 2112, 64) > 0
    assert lib.mrml_moe_dense_ffn_workspace_bytes(0, 2112, 64) == 0
    assert lib.mrml_moe_dense_ffn(2, P, P, P, P, 2816, 2100, 1, P, 1 << 30, None) == -1  # I % 32
    assert lib.mrml_moe_dense_ffn(2, None, P, P, P, 2816, 2112, 1, P, 1 << 30, None) == -1
    assert lib.mrml_moe_dense_ffn(2, P, P, P, P, 2816, 2112, 1, P, 16, None) == -3  # workspace too small
    # Expert-parallel exchange: ranks and shapes are checked first.
    assert lib.mrml_moe_ep_slab_bytes(0, 64, 2816, 8) == 0
    assert lib.mrml_moe_ep_slab_bytes(2, 64, 2818, 8) == 0
    assert lib.mrml_moe_ep_slab_bytes(8, 64, 2816, 8) > 8 * 64 * 2816 * 4
    assert lib.mrml_moe_ep_dispatch(P, 2, 2, 64, 2816, 128, 8, P, P, P, None) == -1  # rank out of range
    assert lib.mrml_moe_ep_dispatch(P, 0, 3, 64, 2816, 128, 8, P, P, P, None) == -1  # E not divisible by N
    assert lib.mrml_moe_ep_combine(None, 0, 2, 64, 2816, 128, 8, P, P, P, P, None) == -1
    assert lib.mrml_moe_ep_workspace_bytes(3, 64, 2816, 704, 128, 8) == 0
    assert lib.mrml_moe_ep_workspace_bytes(8, 64, 2816, 704, 128, 8) > 0
    # the experts step needs the decode kernel's shapes (I a multiple of 64)
    assert lib.mrml_moe_ep_experts(2, P, P, None, P, 0, 2, 64, 2816, 96, 128, 8, P, 1 << 30, None) == -2


def test_zero_tokens_is_a_no_op(moe):
    lib = moe.load_library()
    assert lib.mrml_moe_experts(2, None, None, None, None, None, None, None, 64, 64, 8, 2, 0, None, 0, None) == 0
    assert lib.mrml_moe_router(None, None, None, None, None, 64, 8, 2, 0, None, 0, None) == 0
    assert lib.mrml_moe_experts_shard(2, None, None, None, None, None, None, None, 64, 64, 8, 4, 4, 2, 0, None, 0,
                                      None) == 0
    assert lib.mrml_moe_combine(None, None, None, None, None, None, 64, 2, 0, None) == 0
