"""Writes the golden vectors under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

Inputs are formula-generated (the reference's own test fixtures, restated
from crates/mrml-tensor/src/cuda.rs:3266-3277 and tests/ops_test.rs:459-486)
or seeded synthetic data (qt_llama.cpp_b200/synth.py), so only outputs are
stored.  The GPU tests compare the B200 library with these vectors and with
the oracle run live on the GPU box's host.
"""

from __future__ import annotations

import importlib.util
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def reference_router_fixture():
    """cuda.rs:3266-3277: DIM=257, EXPERTS=128."""
    dim, experts = 257, 128
    x = np.array([((i * 37 % 101) - 50.0) * 0.003 for i in range(dim)], np.float32)
    w = np.array(
        [[(((e * 29 + i * 17) % 113) - 56.0) * 0.002 + e * 0.00001 for i in range(dim)] for e in range(experts)],
        np.float32,
    )
    return x.reshape(1, dim), w, dim, experts


def reference_moe_fixture(oracle):
    """ops_test.rs:459-486: formula-generated Q4_0 experts, H=64, I=32, E=2, K=2."""
    DIM, EXP, EXPERTS = 64, 32, 2
    gate_up = np.zeros((EXPERTS, 2 * EXP, DIM // 32 * 18), np.uint8)
    down = np.zeros((EXPERTS, DIM, EXP // 32 * 18), np.uint8)
    for e in range(EXPERTS):
        for row in range(2 * EXP):
            vals = np.array([(((e * 131 + row * 17 + i * 7) % 101) - 50.0) * 0.002 for i in range(DIM)], np.float32)
            gate_up[e, row] = oracle.quantize(vals, oracle.Q4_0)
        for row in range(DIM):
            vals = np.array([(((e * 97 + row * 19 + i * 11) % 89) - 44.0) * 0.003 for i in range(EXP)], np.float32)
            down[e, row] = oracle.quantize(vals, oracle.Q4_0)
    x = np.array([math.sin(i * 0.031) for i in range(DIM)], np.float32).reshape(1, DIM)
    ids = np.array([[0, 1]], np.int32)
    probs = np.array([[0.65, 0.35]], np.float32)
    scales = np.array([1.0, 0.8], np.float32)
    return dict(gate_up=gate_up, down=down, x=x, ids=ids, probs=probs, scales=scales, H=DIM, I=EXP, E=EXPERTS, K=2)


def c1_inputs(synth, T=4, seed=0):
    """Config 1: H=1024, E=16, K=2, I=512, Q8_0 experts N(0,0.02), router
    N(0,0.02), x N(0,1)."""
    H, I, E, K = 1024, 512, 16, 2
    gu, dn = synth.expert_weights(seed, synth.Q8_0, H, I, E)
    W = synth.normal(seed * 7919 + 11, E * H, 0.02).reshape(E, H)
    x = synth.normal(seed * 7919 + 13, T * H).reshape(T, H)
    return dict(gate_up=gu, down=dn, W=W, x=x, H=H, I=I, E=E, K=K, T=T, wtype=synth.Q8_0)


def _router_case(oracle, synth):
    x, w, dim, experts = reference_router_fixture()
    logits, ids, probs = oracle.router(w, x, dim, experts, 8, 1)
    return dict(logits=logits, ids=ids, probs=probs)


def _moe_case(oracle, synth):
    f = reference_moe_fixture(oracle)
    out = oracle.experts(oracle.Q4_0, f["gate_up"], f["down"], f["ids"], f["probs"], f["scales"], f["x"], f["H"],
                         f["I"], f["E"], f["K"], 1)
    return dict(gate_up=f["gate_up"], down=f["down"], out=out)


def _c1_case(oracle, synth):
    c = c1_inputs(synth)
    logits, ids, probs = oracle.router(c["W"], c["x"], c["H"], c["E"], c["K"], c["T"])
    out = oracle.experts(c["wtype"], c["gate_up"], c["down"], ids, probs, None, c["x"], c["H"], c["I"], c["E"],
                         c["K"], c["T"])
    return dict(logits=logits, ids=ids, probs=probs, out=out)


CASES = {"router_fixture": _router_case, "moe_fixture": _moe_case, "c1_t4": _c1_case}


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
    for name, fn in CASES.items():
        arrays = fn(oracle, synth)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print(name, {k: v.shape for k, v in arrays.items()})
