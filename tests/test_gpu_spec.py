"""Speculative routing of small batches (mrml_moe_forward, T <= 32).

The dispatch selects each token's candidate experts from intervals that
contain the router's logits; the exact router runs on a library-owned stream
beside the expert products and the combine takes its top-K.  Checked here:
  * the intervals contain the oracle's logits (the reference's sequential f32
    chain) on ordinary, cancelling, wide-range, zero and subnormal inputs, and
    are narrow;
  * the layer with speculation on is bit-identical to the oracle and to the
    plain path, at config 2 for every batch up to 32 tokens tried, with
    near ties and exact ties among the top experts (more candidates than K),
    with all logits tied (the dispatch's exact fallback), and under CUDA-graph
    capture and replay.
"""

from __future__ import annotations

import numpy as np
import pytest

from test_gpu_parity import Layer, assert_exact, dev_tensor

pytestmark = pytest.mark.gpu


@pytest.fixture
def spec_on(cuda, moe):
    moe.set_speculative_routing(True)
    yield
    moe.set_speculative_routing(False)


def bounds(moe, cuda, W, x):
    import torch

    T, H = x.shape
    E = W.shape[0]
    lo = torch.empty(T, E, device=cuda)
    hi = torch.empty(T, E, device=cuda)
    moe.router_logit_bounds(dev_tensor(W, cuda), dev_tensor(x, cuda), lo, hi, H, E, T)
    torch.cuda.synchronize()
    return lo.cpu().numpy(), hi.cpu().numpy()


def bound_cases(synth):
    H, E = 2816, 128
    W = synth.normal(501, E * H, 0.02).reshape(E, H)
    x = synth.normal(502, 8 * H).reshape(8, H)
    yield "config2", W, x
    # large cancelling terms: x . w near zero with |x_i w_i| ~ 1
    xc = np.abs(synth.normal(503, 4 * H)).reshape(4, H) + np.float32(1.0)
    Wc = np.tile(np.where(np.arange(H) % 2 == 0, 1.0, -1.0).astype(np.float32), (E, 1))
    Wc += synth.normal(504, E * H, 1e-3).reshape(E, H)
    yield "cancelling", Wc.astype(np.float32), xc.astype(np.float32)
    # wide dynamic range: a few huge inputs among small ones
    xw = synth.normal(505, 4 * H, 1e-3).reshape(4, H)
    xw[:, ::97] = np.float32(3.0e4)
    yield "wide", W, xw
    # zeros
    yield "zeros", np.zeros((16, 256), np.float32), synth.normal(506, 2 * 256).reshape(2, 256)
    # subnormal products
    xs = synth.normal(507, 2 * 512, 1e-20).reshape(2, 512)
    Ws = synth.normal(508, 32 * 512, 1e-20).reshape(32, 512)
    yield "subnormal", Ws, xs


def test_logit_bounds_contain_reference(cuda, moe, oracle, synth):
    for name, W, x in bound_cases(synth):
        T, H = x.shape
        E = W.shape[0]
        lo, hi = bounds(moe, cuda, W, x)
        ref, _, _ = oracle.router(W, x, H, E, 1, T)
        assert np.all(lo <= ref) and np.all(ref <= hi), name
        # narrow: at most about 2 H 2^-24 sum|x_i w_i| wide
        mag = np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
        assert np.all(hi.astype(np.float64) - lo <= 2.5 * (H + 2) * 2.0**-24 * mag + 1e-30), name


def spec_layer_check(moe, cuda, oracle, gu, dn, W, x, H, I, E, K, wtype=2):
    """Forward with speculation on and off: both bit-identical to the oracle."""
    T = x.shape[0]
    L = Layer(moe, cuda, wtype, gu, dn, W, H, I, E, K, T)
    r_logits, r_ids, r_probs = oracle.router(W, x, H, E, K, T)
    ref = oracle.experts(wtype, gu, dn, r_ids, r_probs, None, x, H, I, E, K, T, 8)
    for on in (True, False):
        moe.set_speculative_routing(on)
        ids, probs, out, _ = L.forward(x)
        assert np.array_equal(ids, r_ids)
        assert_exact(L.logits.cpu().numpy(), r_logits)
        assert_exact(probs, r_probs)
        assert_exact(out, ref)
    moe.set_speculative_routing(True)
    return r_logits, r_ids


@pytest.fixture(scope="module")
def c2_small(cuda, moe, synth):
    """Config-2 shapes with 32 experts (the selection and the candidates do
    not depend on the expert count beyond E <= 256)."""
    return synth.expert_weights(61, 2, 2816, 704, 32)


@pytest.mark.parametrize("T", [1, 2, 3, 5, 8, 17, 32])
def test_spec_forward_config2(cuda, moe, oracle, synth, spec_on, c2_small, T):
    H, I, E, K = 2816, 704, 32, 8
    gu, dn = c2_small
    W = synth.normal(62, E * H, 0.02).reshape(E, H)
    x = synth.normal(63 + T, T * H).reshape(T, H)
    spec_layer_check(moe, cuda, oracle, gu, dn, W, x, H, I, E, K)


@pytest.mark.parametrize("T", [2, 16])
def test_spec_near_and_exact_ties(cuda, moe, oracle, synth, spec_on, T):
    """Groups of experts whose router rows differ by about an ulp (logits
    within the intervals' width of one another: more than K candidates) and
    two identical rows (an exact tie, decided by the lower id)."""
    H, I, E, K = 2816, 704, 32, 4
    gu, dn = synth.expert_weights(71, 2, H, I, E)
    base = synth.normal(72, H, 0.02)
    W = np.stack([base + np.float32(1e-7) * synth.normal(73 + e, H) if e % 5 == 0 else synth.normal(90 + e, H, 0.02)
                  for e in range(E)]).astype(np.float32)
    W[10] = base
    W[11] = base
    x = synth.normal(74, T * H).reshape(T, H)
    x += np.float32(4.0) * base[None, :] / np.float32(np.linalg.norm(base))
    r_logits, _ = spec_layer_check(moe, cuda, oracle, gu, dn, W, x, H, I, E, K)
    top = np.sort(r_logits, axis=1)[:, ::-1][:, :K + 1]
    assert (np.diff(top, axis=1) > -1e-4).any()


@pytest.mark.parametrize("T", [1, 2, 9])
def test_spec_all_tied_takes_exact_fallback(cuda, moe, oracle, synth, spec_on, T):
    """A zero router: every logit is 0, every expert a candidate (more than
    the slots), so the dispatch computes the exact logits itself; the top-K
    is experts 0..K-1 with equal weights."""
    H, I, E, K = 2816, 704, 32, 8
    gu, dn = synth.expert_weights(81, 2, H, I, E)
    W = np.zeros((E, H), np.float32)
    x = synth.normal(82 + T, T * H).reshape(T, H)
    _, r_ids = spec_layer_check(moe, cuda, oracle, gu, dn, W, x, H, I, E, K)
    assert np.array_equal(r_ids, np.tile(np.arange(K, dtype=np.int32), (T, 1)))


def test_spec_graph_capture_replay(cuda, moe, oracle, synth, spec_on):
    """The side stream's fork and join are captured with the layer: replays of
    the graph on new inputs give the oracle's results."""
    import torch

    H, I, E, K, T = 2816, 704, 32, 8, 4
    gu, dn = synth.expert_weights(91, 2, H, I, E)
    W = synth.normal(92, E * H, 0.02).reshape(E, H)
    L = Layer(moe, cuda, 2, gu, dn, W, H, I, E, K, T)
    d_x = torch.zeros(T, H, device=cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        moe.forward(2, L.W, d_x, d_x, L.gu, L.dn, None, L.logits, L.ids, L.probs, L.out, H, I, E, K, T, L.ws,
                    stream=s)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        moe.forward(2, L.W, d_x, d_x, L.gu, L.dn, None, L.logits, L.ids, L.probs, L.out, H, I, E, K, T, L.ws,
                    stream=s)
    for seed in (93, 94):
        x = synth.normal(seed, T * H).reshape(T, H)
        d_x.copy_(torch.from_numpy(x))
        g.replay()
        torch.cuda.synchronize()
        assert moe.device_status(L.ws)[0] == 0
        r_logits, r_ids, r_probs = oracle.router(W, x, H, E, K, T)
        ref = oracle.experts(2, gu, dn, r_ids, r_probs, None, x, H, I, E, K, T, 8)
        assert np.array_equal(L.ids.cpu().numpy(), r_ids)
        assert_exact(L.out.cpu().numpy(), ref)
    del g
