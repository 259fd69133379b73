"""The allocation-free router entry point (mrml_moe_router_noalloc).

Callers that cannot allocate device memory (a sandboxed GPU client limited
to buffers it was handed, a latency path that must not allocate, or code
being recorded into a CUDA graph) use this variant: its scratch lives in a
fixed array inside the library.  It must give the same results as the
regular, workspace-taking mrml_moe_router, call after call, even though
every call reuses the same scratch.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _route(moe, fn, W, x, H, E, K, T, device, ws=None):
    import torch

    logits = torch.full((T, E), float("nan"), device=device)
    ids = torch.full((T, K), -1, dtype=torch.int32, device=device)
    probs = torch.full((T, K), float("nan"), device=device)
    if ws is None:
        fn(W, x, logits, ids, probs, H, E, K, T)
    else:
        fn(W, x, logits, ids, probs, H, E, K, T, ws)
    torch.cuda.synchronize()
    return logits.cpu().numpy(), ids.cpu().numpy(), probs.cpu().numpy()


def test_noalloc_router_matches_workspace_router_on_consecutive_calls(cuda, moe, synth):
    import torch

    H, E, K = 2816, 128, 8
    W = torch.from_numpy(synth.normal(301, E * H, 0.02).reshape(E, H)).to(cuda)
    ws = moe.new_workspace(32, 32, E, K, 64, cuda)
    # Two calls in a row with different token counts and inputs: the second
    # call must not see anything the first one left in the shared scratch.
    for call, T in enumerate((64, 9)):
        x = torch.from_numpy(synth.normal(400 + call, T * H).reshape(T, H)).to(cuda)
        ref = _route(moe, moe.router, W, x, H, E, K, T, cuda, ws)
        got = _route(moe, moe.router_noalloc, W, x, H, E, K, T, cuda)
        assert np.array_equal(got[1], ref[1]), f"call {call}: expert ids differ"
        # Same kernels on the same inputs: logits and probabilities agree to
        # the bit, well inside the router tolerance of 2e-5.
        assert np.abs(got[2] - ref[2]).max() <= 2e-5
        assert np.abs(got[0] - ref[0]).max() <= 2e-5
        assert np.array_equal(got[2], ref[2]) and np.array_equal(got[0], ref[0])


def test_noalloc_router_at_the_size_limit(cuda, moe, synth):
    """T * E exactly at the fixed limit (512 x 128 = 65536): accepted, runs the
    large-batch (tiled) logits kernel, and matches the workspace router bit
    for bit; the status reader then reports no device-side failure."""
    import torch

    H, E, K, T = 2816, 128, 8, 512
    W = torch.from_numpy(synth.normal(302, E * H, 0.02).reshape(E, H)).to(cuda)
    x = torch.from_numpy(synth.normal(402, T * H).reshape(T, H)).to(cuda)
    ws = moe.new_workspace(32, 32, E, K, T, cuda)
    ref = _route(moe, moe.router, W, x, H, E, K, T, cuda, ws)
    got = _route(moe, moe.router_noalloc, W, x, H, E, K, T, cuda)
    assert np.array_equal(got[1], ref[1])
    assert np.array_equal(got[2], ref[2]) and np.array_equal(got[0], ref[0])
    lib = moe.load_library()
    assert lib.mrml_moe_router_noalloc_status(None) == 0
    assert lib.mrml_moe_router_noalloc_status(None) == 0  # reading clears; still clean


def test_noalloc_router_rejects_oversized_batches(cuda, moe):
    lib = moe.load_library()
    P = ctypes.c_void_p(0x1000)
    # T * E above the fixed scratch (65536 bounds): a clear error, no launch.
    st = lib.mrml_moe_router_noalloc(P, P, P, P, P, 1024, 128, 8, 513, None)
    assert st == -2
    assert lib.mrml_moe_status_string(st) == b"unsupported shape or weight type"
