"""Benchmark of the B200 MoE FFN layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

A step is one MoE layer (router logits, top-k/softmax, dispatch, grouped
gate/up + GeGLU, down, weighted combine) over one batch of T tokens, through
the library's public C ABI (mrml_moe_forward).  The headline workload is
config 2 of the task (Gemma-4-26B-A4B MoE shape: H=2816, E=128, K=8, I=704,
Q4_0 experts) at decode batch T=64; T=1, T=8 and the config-3 prefill
(H=1024, E=16, K=2, I=512, Q8_0, T=2048, Zipf-skewed logits) are reported
under "also".  Data are synthetic (seeded N(0,0.02) weights quantised with
the reference's rules, N(0,1) activations).

Timing: W untimed warm-up steps, then K steps between CUDA events on the
launch stream, bracketed by a barrier and torch.cuda.synchronize(); the
max over ranks is reported.  Consecutive steps rotate over independent layer
copies whose weights together exceed the 126 MB L2, so every step streams its
experts from HBM.  `value` is tokens/s with inputs resident in HBM; `e2e`
adds, every step, the host->device copy of x from pinned memory and the
device->host copy of the layer output.

With --gpus N > 1 (torchrun, one rank per GPU) the layer runs expert-
parallel: rank r holds experts [r*E/N, (r+1)*E/N) and 64 home tokens (weak
scaling: N*64 tokens per step); a step routes the home tokens, sends them to
every rank, runs the rank's experts on every rank's tokens and returns the
partial outputs to their home ranks (qt_llama.cpp_b200/ep.py): by default
with the library's peer-memory kernels over NVLink (--ep-exchange p2p), or
with NCCL all-gathers and a reduce-scatter (--ep-exchange nccl).  Workload
"c4" is config 4: 8192 tokens per step in total (strong scaling); "c5" is
config 5: a 30-layer stack with an RMS norm between layers, 32 tokens.

--impl reference times the reference's CPU algorithm (the C restatement
under oracle/, the reference's Rust cannot be built here) on the host cores.
"""

from __future__ import annotations

import argparse
import gc
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 1024 * 1024


def _load(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def package():
    moe = _load("mrml_moe_b200", os.path.join(ROOT, "qt_llama.cpp_b200", "mrml_moe.py"))
    synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
    return moe, synth


WORKLOADS = {
    # name: (wtype, H, I, E, K, T, routing); T is per rank, except for the
    # STRONG workloads, whose T is the whole job's (T / N home tokens per rank).
    "c2_t64": (2, 2816, 704, 128, 8, 64, "router"),
    "c2_t8": (2, 2816, 704, 128, 8, 8, "router"),
    "c2_t1": (2, 2816, 704, 128, 8, 1, "router"),
    "c2_t16": (2, 2816, 704, 128, 8, 16, "router"),
    "c2_t32": (2, 2816, 704, 128, 8, 32, "router"),
    "c3_prefill": (8, 1024, 512, 16, 2, 2048, "zipf_logits"),
    "c1_t4": (8, 1024, 512, 16, 2, 4, "router"),
    "c2_t512": (2, 2816, 704, 128, 8, 512, "router"),
    "c3_c2q8": (8, 2816, 704, 128, 8, 2048, "zipf_logits"),
    "c4": (2, 2816, 704, 128, 8, 8192, "router"),
    "c4_q8": (8, 2816, 704, 128, 8, 8192, "router"),
}
STRONG = {"c4", "c4_q8"}
METRIC = "MoE-layer tokens/sec at decode batch 1/64 and 2048-token prefill; % of roofline"
KERNELS = {
    "router": ["router_logits", "router_topk", "dispatch", "quantize", "gate_up", "down", "combine"],
    # mrml_moe_forward at most 32 tokens (E <= 256, K <= 64): the dispatch
    # kernel selects the experts itself (the library's dispatch_topk_supported)
    "router_small": ["router_logits", "topk_dispatch", "quantize", "gate_up", "down", "combine"],
    # speculative routing (--spec 1, up to 32 tokens when H % 128 == 0 and
    # K < E): the exact router on the library's side stream, the intervals
    # and the candidate dispatch on the caller's
    "router_spec": ["router_logits", "router_topk", "router_bounds", "spec_dispatch", "quantize", "gate_up", "down",
                    "combine"],
    "zipf_logits": ["route_from_logits", "dispatch", "quantize", "gate_up", "down", "combine"],
}


def expert_kernels(T):
    """Launch list of the expert products for T tokens on the decode kernels:
    from 256 tokens the input is quantised per token, then gathered per
    position group after the dispatch (the library's kGatherMinTokens)."""
    if T >= 256:
        return ["quantize_rows", "dispatch", "gather", "gate_up", "down", "combine"]
    return ["dispatch", "quantize", "gate_up", "down", "combine"]


SPEC = {"on": False}  # --spec


def forward_kernels(T, E, K, H=2816):
    """Launch list of one mrml_moe_forward call."""
    if T <= 32 and E <= 256 and K <= 64:
        spec = SPEC["on"] and H % 128 == 0 and K < E
        return KERNELS["router_spec"] if spec else KERNELS["router_small"]
    return ["router_logits", "router_topk"] + expert_kernels(T)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def int8_peak_tops():
    """Dense int8 tensor peak used for the prefill roofline.  MEASURED_PEAKS
    holds the measured dense bf16 GEMM rate; B200's dense int8 rate is twice
    its bf16 rate (4.5 vs 2.25 POPS nominal), so the peak is derived as 2x the
    measured bf16 burst figure (fallback: 2 x 1590 TFLOP/s)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return 2.0 * float(json.load(f)["bf16_tflops"]), "derived: 2 x measured dense bf16 (MEASURED_PEAKS.json)"
    except Exception:
        return 2.0 * 1590.0, "derived: 2 x fallback dense bf16 1590 TFLOP/s"


def int8_ops(ls, pairs):
    """int8 multiply-add operations (2 per MAC) of the expert products for
    `pairs` (token, slot) pairs: gate/up 2I x H and down H x I per pair."""
    return 2 * pairs * (2 * ls.I * ls.H + ls.H * ls.I), 2 * pairs * (2 * ls.I * ls.H)


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    every few milliseconds (the timed regions are short), else nvidia-smi."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits, in the order of FIELDS[2:].
    NVML_BITS = (0x8, 0x40, 0x20, 0x4)

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
                h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self._nvml = (pynvml, h)
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        nv, h = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        return [str(sm), str(mx)] + ["Active" if bits & b else "Not Active" for b in self.NVML_BITS]

    def _run(self):
        while not self._stop.is_set():
            try:
                if self._nvml is not None:
                    self.samples.append(self._sample_nvml())
                    self._stop.wait(0.005)
                    continue
                out = subprocess.run(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.gpu)],
                    capture_output=True, text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([v.strip() for v in out.split(",")])
            except Exception:
                self._nvml = None
            self._stop.wait(0.1)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 2 + i and s[2 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples),
                "source": "nvml" if self._nvml is not None else "nvidia-smi"}


class LayerSet:
    """Independent copies of one MoE layer on the device (weights + router),
    enough of them that their weights exceed L2, plus per-step inputs."""

    def __init__(self, moe, synth, device, name, n_inputs, seed=0, packed=False):
        import torch

        wtype, H, I, E, K, T, routing = WORKLOADS[name]
        self.moe, self.device, self.name = moe, device, name
        self.wtype, self.H, self.I, self.E, self.K, self.T, self.routing = wtype, H, I, E, K, T, routing
        # the weight type passed to the library: packed weights carry the flag
        self.wcall = wtype | (moe.MRML_PACKED if packed else 0)
        bb = 18 if wtype == 2 else 34
        layer_bytes = E * (2 * I * (H // 32) * bb + H * (I // 32) * bb)
        self.n_layers = max(2, -(-4 * L2_BYTES // layer_bytes))
        self.layers = []
        self.host_layer0 = None
        for l in range(self.n_layers):
            gu, dn = synth.expert_weights_device(seed * 100 + l + 1, wtype, H, I, E, device, moe.quantize)
            g = torch.Generator(device=device)
            g.manual_seed(seed * 100 + l + 1000)
            W = torch.randn((E, H), generator=g, device=device).mul_(0.02)
            if l == 0:  # the parity check's reference weights (GGUF layout)
                self.host_layer0 = (gu.cpu().numpy(), dn.cpu().numpy(), W.cpu().numpy())
            if packed:  # the load-time repack (mrml_moe_prepare_weights), outside the timed steps
                gu, dn = moe.prepare_weights(wtype, gu, dn)
                torch.cuda.synchronize()
            self.layers.append((gu, dn, W))
        g = torch.Generator(device=device)
        g.manual_seed(seed + 77)
        self.xs = [torch.randn((T, H), generator=g, device=device) for _ in range(n_inputs)]
        if routing == "zipf_logits":
            bias = torch.from_numpy(synth.zipf_bias(seed + 5, E)).to(device)
            self.logit_in = [torch.randn((T, E), generator=g, device=device) + bias[None, :] for _ in range(n_inputs)]
        self.logits = torch.empty(T, E, device=device)
        self.ids = torch.empty(T, K, dtype=torch.int32, device=device)
        self.probs = torch.empty(T, K, device=device)
        self.out = torch.empty(T, H, device=device)
        self.ws = moe.new_workspace(H, I, E, K, T, device)
        self.layer_bytes = layer_bytes
        self.kernels = forward_kernels(T, E, K, H) if routing == "router" else ["route_from_logits"] + expert_kernels(T)

    def step(self, i, x=None, out=None):
        gu, dn, W = self.layers[i % self.n_layers]
        x = self.xs[i % len(self.xs)] if x is None else x
        out = self.out if out is None else out
        m = self.moe
        if self.routing == "router":
            m.forward(self.wcall, W, x, x, gu, dn, None, self.logits, self.ids, self.probs, out, self.H, self.I,
                      self.E, self.K, self.T, self.ws)
        else:
            m.route_from_logits(self.logit_in[i % len(self.logit_in)], self.ids, self.probs, self.E, self.K, self.T)
            m.experts(self.wcall, gu, dn, self.ids, self.probs, None, x, out, self.H, self.I, self.E, self.K, self.T,
                      self.ws)

    def capture(self, i, profile_events=None):
        """A CUDA graph of step i (the decode path replays per-layer graphs, as
        the reference's capture_layer_ffn_graph does, model.rs:295-381).  With
        profile_events, the library's hook records them around every launch."""
        import ctypes

        import torch

        lib = self.moe.load_library()
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.step(i)  # warm the host-side caches outside capture
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=side):
            if profile_events is not None:
                handles = (ctypes.c_void_p * len(profile_events))(*[e.cuda_event for e in profile_events])
                assert lib.mrml_moe_profile_events(handles, len(profile_events)) == 0
            try:
                self.step(i)
            finally:
                lib.mrml_moe_profile_events(None, 0)
        return g

    def n_kernels(self):
        return len(self.kernels)

    @property
    def router_ws(self):
        return self.ws

    def unique_experts(self, i):
        """Experts hit (with alpha > 1e-4) by step i's routing, and the pair count."""
        self.step(i)
        ids = self.ids.cpu().numpy()
        probs = self.probs.cpu().numpy()
        hit = ids[probs > 1e-4]
        return len(np.unique(hit)), int(hit.size)


class EPLayerSet:
    """The expert-parallel layer on this rank: every layer copy holds the
    rank's E/N experts and the replicated router; a step routes the rank's
    home tokens, sends each row only to the ranks that own one of its experts,
    runs the rank's experts on the rows it received and returns the partial
    outputs to their home ranks (qt_llama.cpp_b200/ep.py).  Same interface as
    LayerSet."""

    def __init__(self, moe, synth, device, name, n_inputs, rank, world, seed=0, exchange="p2p", packed=False):
        import torch

        self.epm = ep = _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))
        wtype, H, I, E, K, T, routing = WORKLOADS[name]
        assert routing == "router", "expert parallelism runs the router workloads"
        if name in STRONG:
            T //= world
        self.moe, self.device, self.name = moe, device, name
        self.wtype, self.H, self.I, self.E, self.K, self.T, self.routing = wtype, H, I, E, K, T, routing
        self.world, self.rank, self.exchange = world, rank, exchange
        wcall = wtype | (moe.MRML_PACKED if packed else 0)
        self.ep = ep.ExpertParallelLayer(moe, rank, world, wcall, H, I, E, K, T, device, exchange=exchange)
        first, count = self.ep.first, self.ep.count
        bb = 18 if wtype == 2 else 34
        layer_bytes = count * (2 * I * (H // 32) * bb + H * (I // 32) * bb)
        self.n_layers = max(2, -(-4 * L2_BYTES // layer_bytes))
        self.layers = []
        self.host_layer0 = None
        for l in range(self.n_layers):
            # Every rank generates the whole layer with the same seed and keeps
            # its experts, so that the job computes one well-defined layer.
            gu, dn = synth.expert_weights_device(seed * 100 + l + 1, wtype, H, I, E, device, moe.quantize)
            g = torch.Generator(device=device)
            g.manual_seed(seed * 100 + l + 1000)
            W = torch.randn((E, H), generator=g, device=device).mul_(0.02)
            if l == 0 and rank == 0:  # the parity check's reference weights (GGUF layout)
                self.host_layer0 = (gu.cpu().numpy(), dn.cpu().numpy(), W.cpu().numpy())
            gu, dn = gu[first:first + count].clone(), dn[first:first + count].clone()
            if packed:
                gu, dn = moe.prepare_weights(wtype, gu, dn)
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            self.layers.append((gu, dn, W))
        g = torch.Generator(device=device)
        g.manual_seed(seed + 77 + 1000 * rank)
        self.xs = [torch.randn((T, H), generator=g, device=device) for _ in range(n_inputs)]
        self.out = torch.empty(T, H, device=device)
        self.ids, self.probs = self.ep.ids, self.ep.probs
        self.ws = self.ep.ws
        self.layer_bytes = layer_bytes
        if self.ep.exchange == "p2p":
            # router on the home tokens; push; then the expert step (receive,
            # dispatch, gather, gate/up, down, partials pushed home); reduce
            self.kernels = ["router_logits", "router_topk", "ep_push", "ep_recv", "dispatch", "gather", "gate_up",
                            "down", "ep_combine_push", "ep_reduce"]
        else:  # router, then the expert shard on all ranks' tokens (NCCL moves the data)
            self.kernels = ["router_logits", "router_topk"] + expert_kernels(T * world)

    @property
    def router_ws(self):
        return self.ep.router_ws

    def step(self, i, x=None, out=None):
        gu, dn, W = self.layers[i % self.n_layers]
        x = self.xs[i % len(self.xs)] if x is None else x
        out = self.out if out is None else out
        self.ep.forward(W, x, gu, dn, out)

    capture = LayerSet.capture

    def n_kernels(self):
        return len(self.kernels)

    def gather_routing(self):
        """Every rank's home ids and weights of the last step, rank order."""
        ids = all_gather_np(self.ids, self.world)
        probs = all_gather_np(self.probs, self.world)
        return ids, probs

    def unique_experts(self, i):
        """This rank's experts hit by step i (every rank's tokens) and its
        pair count; also keeps step i's routing for nvlink_bytes."""
        self.step(i)
        ids, probs = self.gather_routing()
        self._routing = (ids, probs)
        first, count = self.ep.first, self.ep.count
        hit = ids[(probs > 1e-4) & (ids >= first) & (ids < first + count)]
        return len(np.unique(hit)), int(hit.size)

    def nvlink_bytes(self):
        """Bytes this rank receives per step.  Peer exchange: the Q8_0 rows of
        the tokens routed to its experts, every rank's ids and weights, and
        the partials of its home tokens from the ranks that own their experts
        (counted from the routing of the step unique_experts ran).  NCCL
        baseline: the all-gathers bring (N-1) home batches of f32 rows, ids and
        weights; the reduce-scatter moves (N-1)/N of the [N*T, H] partials."""
        n, T, H, K = self.world, self.T, self.H, self.K
        if self.ep.exchange == "p2p":
            ids, probs = self._routing
            return self.epm.exchange_bytes(ids, probs, n, self.E, H, K, self.rank, T)["total"]
        return (n - 1) * T * (H * 4 + K * 8) + (n - 1) * T * H * 4

    def close(self):
        self.ep.close()


def all_gather_np(t, world):
    """A device tensor's values from every rank, concatenated in rank order
    along the first axis (host numpy); the tensor itself at world 1."""
    import torch

    if world == 1:
        return t.cpu().numpy()
    import torch.distributed as dist

    buf = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(buf, t.contiguous())
    return buf.cpu().numpy()


def parity_check(ls, world, rank, n_check=64, seed=123):
    """One step outside the timed region, checked against the oracle (the
    reference's CPU path) on a seeded sample of the job's tokens: their
    expert ids must be identical, their outputs within the task's bars
    (max-abs <= 1e-3 * max|ref|, rel-L2 <= 1e-4).  Every rank takes part (the
    step and the gathers); rank 0 computes and returns the record."""
    import torch

    oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    x = ls.xs[0]
    ls.step(0, x=x)
    torch.cuda.synchronize()
    xs = all_gather_np(x, world)
    outs = all_gather_np(ls.out, world)
    ids = all_gather_np(ls.ids, world)
    if rank != 0:
        return None
    gu, dn, W = ls.host_layer0
    H, I, E, K = ls.H, ls.I, ls.E, ls.K
    idx = np.sort(np.random.default_rng(seed).choice(xs.shape[0], size=min(n_check, xs.shape[0]), replace=False))
    n = len(idx)
    if ls.routing == "router":
        _, r_ids, r_probs = oracle.router(W, xs[idx], H, E, K, n)
    else:
        r_ids, r_probs = oracle.route_from_logits(ls.logit_in[0].cpu().numpy()[idx], E, K, n)
    ref = oracle.experts(ls.wtype, gu, dn, r_ids, r_probs, None, xs[idx], H, I, E, K, n, os.cpu_count() or 1)
    got = outs[idx].astype(np.float64)
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    mx = float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
    ids_ok = bool(np.array_equal(ids[idx], r_ids))
    return {"ok": ids_ok and rel <= 1e-4 and mx <= 1e-3, "ids_exact": ids_ok, "max_rel_l2": rel,
            "max_abs_frac": mx, "bit_exact": bool(np.array_equal(outs[idx], ref)), "tokens_checked": n,
            "of_tokens": int(xs.shape[0]), "reference": "oracle/ (the reference's CPU MoE path restated)"}


class StackSet:
    """Config 5: a stack of 30 independent MoE FFN blocks of the config-2
    shape (Q4_0), decode batch of 32 tokens in total, each block as a Gemma-4
    layer runs its FFN half without the attention and the shared MLP: the
    fused prologue (model.rs:1719-1784: router input and experts' input, two
    RMS norms of h), the MoE layer, and the fused epilogue (model.rs:
    2176-2196: post-norms, residual add, layer scale) producing h_{l+1}.  With N > 1 every layer runs expert-parallel (T = 32/N
    home tokens per rank), one exchange object shared by the 30 layers.
    A step runs the whole stack; inputs are fresh N(0,1) batches."""

    N_LAYERS = 30

    def __init__(self, moe, synth, device, n_inputs, rank, world, exchange="p2p", seed=0, packed=False):
        import torch

        ep = _load("mrml_moe_b200_ep", os.path.join(ROOT, "qt_llama.cpp_b200", "ep.py"))
        wtype, H, I, E, K = 2, 2816, 704, 128, 8
        self.wcall = wtype | (moe.MRML_PACKED if packed else 0)
        T = 32 // world
        self.moe, self.device, self.name = moe, device, "c5"
        self.wtype, self.H, self.I, self.E, self.K, self.T, self.routing = wtype, H, I, E, K, T, "router"
        self.world = world
        self.n_layers = 1  # graphs per input: one graph holds the whole stack
        if world > 1:
            self.ep = ep.ExpertParallelLayer(moe, rank, world, self.wcall, H, I, E, K, T, device, exchange=exchange)
            first, count = self.ep.first, self.ep.count
        else:
            self.ep = None
            first, count = 0, E
            self.ws = moe.new_workspace(H, I, E, K, T, device)
            self.logits = torch.empty(T, E, device=device)
            self.ids = torch.empty(T, K, dtype=torch.int32, device=device)
            self.probs = torch.empty(T, K, device=device)
        self.layers = []
        for l in range(self.N_LAYERS):
            gu, dn = synth.expert_weights_device(seed * 1000 + 500 + l, wtype, H, I, E, device, moe.quantize)
            if world > 1:
                gu, dn = gu[first:first + count].clone(), dn[first:first + count].clone()
                torch.cuda.empty_cache()
            if packed:
                gu, dn = moe.prepare_weights(wtype, gu, dn)
                torch.cuda.synchronize()
            g = torch.Generator(device=device)
            g.manual_seed(seed * 1000 + 900 + l)
            W = torch.randn((E, H), generator=g, device=device).mul_(0.02)
            # norm weights of the block: pre_ffw_norm_2, router scale, post_ffw_norm_2, post_ffw_norm
            norms = [torch.randn(H, generator=g, device=device).mul_(0.1).add_(1.0) for _ in range(4)]
            self.layers.append((gu, dn, W, norms))
        self.seed = seed
        bb = 18
        self.layer_bytes = count * (2 * I * (H // 32) * bb + H * (I // 32) * bb)
        g = torch.Generator(device=device)
        g.manual_seed(seed + 77 + 1000 * rank)
        self.xs = [torch.randn((T, H), generator=g, device=device) for _ in range(n_inputs)]
        self.h = [torch.empty((T, H), device=device) for _ in range(2)]
        self.moe_out = torch.empty((T, H), device=device)
        self.x_moe = torch.empty((T, H), device=device)
        self.router_x = torch.empty((T, H), device=device)
        self.out = torch.empty((T, H), device=device)

    def step(self, i, x=None, out=None):
        m, H, T = self.moe, self.H, self.T
        h = self.xs[i % len(self.xs)] if x is None else x
        out = self.out if out is None else out
        for l in range(len(self.layers)):
            nxt = out if l == len(self.layers) - 1 else self.h[l & 1]
            self.layer_step(l, h, nxt)
            h = nxt

    def layer_step(self, l, h, nxt):
        """Block l on h (the same calls as step)."""
        m, H, T = self.moe, self.H, self.T
        gu, dn, W, (pre2, rscale, post2, post) = self.layers[l]
        m.ffn_prologue(h, None, None, None, pre2, rscale, None, None, self.x_moe, self.router_x, H, T)
        if self.ep is not None:
            self.ep.forward(W, self.x_moe, gu, dn, self.moe_out, router_x=self.router_x)
        else:
            m.forward(self.wcall, W, self.router_x, self.x_moe, gu, dn, None, self.logits, self.ids, self.probs,
                      self.moe_out, H, self.I, self.E, self.K, T, self.ws)
        m.ffn_epilogue(h, None, self.moe_out, None, post2, post, nxt, 1.0, H, T)

    def raw_layer_host(self, l):
        """Layer l's GGUF-layout expert slabs (all E experts) on the host,
        regenerated from the layer's seed."""
        import torch

        synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
        gu, dn = synth.expert_weights_device(self.seed * 1000 + 500 + l, self.wtype, self.H, self.I, self.E,
                                             self.device, self.moe.quantize)
        out = gu.cpu().numpy(), dn.cpu().numpy()
        del gu, dn
        torch.cuda.empty_cache()
        return out

    capture = LayerSet.capture

    def n_kernels(self):
        return 0


def stack_parity_check(ss, world, rank, layers=(0, 1, 29), n_check=4, seed=321):
    """Config 5 outside the timed region: the stack runs block by block on
    one input, and for each block in `layers` the oracle (the reference's CPU
    FFN block, model.rs:1719-1784, 1804-1829, 2111-2196) recomputes a seeded
    sample of tokens from the same block input; ids and outputs must be
    identical.  Every rank takes part; rank 0 returns the record."""
    import torch

    oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    H, I, E, K = ss.H, ss.I, ss.E, ss.K
    h = ss.xs[0].clone()
    nxt = torch.empty_like(h)
    saved = {}
    for l in range(len(ss.layers)):
        ss.layer_step(l, h, nxt)
        if l in layers:
            torch.cuda.synchronize()
            ids = ss.ep.ids if ss.ep is not None else ss.ids
        saved[l] = (all_gather_np(h, world), all_gather_np(nxt, world), all_gather_np(ids, world))
        h, nxt = nxt, h
    exact, worst, worst_abs, n_ids_bad = True, 0.0, 0.0, 0
    idx = None
    for l in layers:
        # every rank regenerates in step (the quantiser runs on each device);
        # only rank 0 checks
        gu, dn = ss.raw_layer_host(l)
        if rank != 0:
            continue
        x, y, ids = saved[l]
        if idx is None:
            idx = np.sort(np.random.default_rng(seed).choice(x.shape[0], size=min(n_check, x.shape[0]),
                                                             replace=False))
        W = ss.layers[l][2].cpu().numpy()
        pre2, rscale, post2, post = [w.cpu().numpy() for w in ss.layers[l][3]]
        _, _, xm, rx = oracle.ffn_prologue(x[idx], None, None, None, pre2, rscale)
        _, r_ids, r_probs = oracle.router(W, rx, H, E, K, len(idx))
        moe_raw = oracle.experts(ss.wtype, gu, dn, r_ids, r_probs, None, xm, H, I, E, K, len(idx),
                                 os.cpu_count() or 1)
        ref = oracle.ffn_epilogue(x[idx], None, moe_raw, None, post2, post, 1.0)
        got = y[idx]
        n_ids_bad += int(np.count_nonzero(np.any(ids[idx] != r_ids, axis=1)))
        rel = float(np.linalg.norm(got.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30))
        mx = float(np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))
        worst, worst_abs = max(worst, rel), max(worst_abs, mx)
        exact = exact and bool(np.array_equal(got, ref))
    if rank != 0:
        return None
    # the task's bars (ids exact, max-abs <= 1e-3 max|ref|, rel-L2 <= 1e-4); under
    # expert parallelism the rank-order sum of partials is not bit-identical
    ok = n_ids_bad == 0 and worst <= 1e-4 and worst_abs <= 1e-3
    return {"ok": ok, "bit_exact": exact, "ids_exact": n_ids_bad == 0, "max_rel_l2": worst, "max_abs_frac": worst_abs,
            "layers_checked": list(layers), "tokens_checked_per_layer": int(len(idx)),
            "reference": "oracle/ (the reference's CPU FFN block restated)"}


def run_stack(args):
    """Config 5 through the public API (see StackSet); prints the JSON line."""
    import torch

    rank, world, local = dist_setup(args.gpus)
    moe, synth = package()
    device = torch.device("cuda", local)
    moe.load_library()
    hbm_peak, peak_kind = peaks()
    ss = StackSet(moe, synth, device, 4, rank, world, exchange=args.ep_exchange, packed=args.weights == "packed")
    graphs = [ss.capture(g) for g in range(2)]
    reps = repeats_for(ss, args.steps, args.warmup, world, graphs, target_s=1.0, cap=20)
    with ClockSampler(local) as clk:
        ms = time_steps(ss, args.steps, args.warmup, world, graphs, reps)
    del graphs
    e2e_ms, h2d, d2h = time_e2e(ss, args.steps, args.warmup, world)
    total_tokens = world * ss.T
    step_ms = ms / args.steps
    nl = StackSet.N_LAYERS
    # Per layer at 32 tokens about 200 of the 256 (token, slot) pairs hit
    # distinct experts; the bytes counted are the rank's expert slabs touched
    # (an upper bound of the algorithmic bytes) plus the router weights.
    layer_bytes = ss.layer_bytes + ss.E * ss.H * 4
    line = {
        "metric": METRIC,
        "value": round(total_tokens * args.steps / (ms / 1e3), 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4_0 weights x q8_0 activations, int32 block dots, f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights quantised with the reference's Q4_0 rules, fresh N(0,1) x)",
        "config": {"workload": "c5", "layers": nl, "hidden": ss.H, "experts": ss.E, "top_k": ss.K,
                   "expert_ffn": ss.I, "tokens_per_step": total_tokens, "home_tokens_per_rank": ss.T,
                   "block": "fused FFN prologue (pre_ffw_norm_2, router input) + MoE + fused epilogue "
                            "(post-norms, residual), model.rs:1719-1784 and 2176-2196",
                   "parallelism": (f"ep{world} (" + args.ep_exchange + " exchange)") if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: each step streams {nl} layers "
                         f"({nl * ss.layer_bytes / 1e6:.0f} MB of this rank's expert weights)"},
        "layer_roofline": {"achieved": round(nl * layer_bytes / (step_ms / 1e3) / 1e9, 1), "peak": hbm_peak,
                           "unit": "GB/s", "frac": round(nl * layer_bytes / (step_ms / 1e3) / 1e9 / hbm_peak, 4),
                           "bytes_per_step_upper_bound": nl * layer_bytes, "peak_source": peak_kind},
        "e2e": {"value": round(total_tokens * args.steps / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        # per layer: the MoE launches (forward at world 1; router, expert
        # shard and the exchange kernels under expert parallelism) + the
        # prologue and epilogue
        "gpu_launches": args.steps * nl * (2 + (len(forward_kernels(ss.T, ss.E, ss.K, ss.H)) if world == 1 else
                                               (11 if args.ep_exchange == "p2p" else 7))),
        "clocks": clk.summary(),
    }
    line["parity"] = stack_parity_check(ss, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import gc

        import torch.distributed as dist

        gc.collect()
        torch.cuda.synchronize()
        ss.ep.close()
        dist.destroy_process_group()


def dist_setup(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(ls, steps, warmup, world, graphs, repeats=1, stats=None):
    """Device time (ms) of `steps` consecutive graph replays after `warmup`.

    The K-step region (bracketed by a barrier and a synchronize on both sides,
    CUDA events on the replay stream, max over ranks) is measured `repeats`
    times back to back and the median is returned, so that a short region is
    seen by many clock samples; `stats` (a dict) receives every repeat."""
    import torch

    G = len(graphs)
    for i in range(warmup):
        graphs[i % G].replay()
    s = torch.cuda.current_stream()
    times = []
    for r in range(repeats):
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(steps):
            graphs[(warmup + i) % G].replay()
        e1.record(s)
        torch.cuda.synchronize()
        barrier(world)
        times.append(max_over_ranks(e0.elapsed_time(e1), world))
    if stats is not None:
        stats["repeats"] = repeats
        stats["ms_min"], stats["ms_max"] = round(min(times), 5), round(max(times), 5)
    return statistics.median(times)


def repeats_for(ls, steps, warmup, world, graphs, target_s=0.3, cap=200):
    """Repeats of the K-step region that fill about `target_s` seconds (at
    least 5; same count on every rank)."""
    one = time_steps(ls, steps, warmup, world, graphs)
    return int(min(cap, max(5, target_s * 1e3 / max(one, 1e-3))))


def time_kernels(ls, steps):
    """Per-kernel device times (ms, summed over steps): graphs captured with
    the library's profiling hook, which records events around every launch on
    the stream the kernels run on; one graph replay per step."""
    import torch

    nk = ls.n_kernels()
    totals = [0.0] * nk
    G = min(steps, 2 * ls.n_layers)
    prof = []
    for g in range(G):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * nk)]
        for e in evs:
            e.record()
        torch.cuda.synchronize()
        prof.append((ls.capture(g, evs), evs))
    for i in range(steps):
        graph, evs = prof[i % G]
        graph.replay()
        torch.cuda.synchronize()
        for k in range(nk):
            totals[k] += evs[2 * k].elapsed_time(evs[2 * k + 1])
    return dict(zip(ls.kernels, totals))


def time_e2e(ls, steps, warmup, world, repeats=5):
    """Same steps through the public API with host buffers: every step copies
    its x from pinned host memory to the device, runs the layer and copies the
    output back to pinned host memory.  Steps are independent batches, so the
    copies run on two copy streams (in, out) and overlap the neighbouring
    steps' compute (double-buffered device x and output, events between the
    streams): step i's input copy overlaps step i-1's layer, its output copy
    step i+1's.  The
    `steps` steps are captured as one CUDA graph (the reference's decode path
    captures its per-layer FFN work; one graph keeps the host out of the
    loop), replayed `repeats` times after `warmup` replays of the graph; the
    region is one replay (events, synchronize and barrier around it), median,
    max over ranks."""
    import torch

    T, H = ls.T, ls.H
    G = 2 * ls.n_layers
    host_x = [ls.xs[g % len(ls.xs)].cpu().pin_memory() for g in range(G)]
    host_out = [torch.empty((T, H), dtype=torch.float32).pin_memory() for _ in range(G)]
    dx = [torch.empty((T, H), device=ls.device) for _ in range(2)]
    dout = [torch.empty((T, H), device=ls.device) for _ in range(2)]
    comp = torch.cuda.Stream(device=ls.device)
    cin, cout = torch.cuda.Stream(device=ls.device), torch.cuda.Stream(device=ls.device)
    x_ready = [torch.cuda.Event() for _ in range(2)]
    y_ready = [torch.cuda.Event() for _ in range(2)]
    x_free = [torch.cuda.Event() for _ in range(2)]
    y_free = [torch.cuda.Event() for _ in range(2)]
    fork, join_in, join_out = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()

    def run(n):
        fork.record(comp)
        cin.wait_event(fork)
        cout.wait_event(fork)
        for i in range(n):
            b = i & 1
            if i >= 2:
                cin.wait_event(x_free[b])  # step i-2's layer has read dx[b]
            with torch.cuda.stream(cin):
                dx[b].copy_(host_x[i % G], non_blocking=True)
            x_ready[b].record(cin)
            comp.wait_event(x_ready[b])
            if i >= 2:
                comp.wait_event(y_free[b])  # step i-2's output copy has read dout[b]
            with torch.cuda.stream(comp):
                ls.step(i % G, x=dx[b], out=dout[b])
            x_free[b].record(comp)
            y_ready[b].record(comp)
            cout.wait_event(y_ready[b])
            with torch.cuda.stream(cout):
                host_out[i % G].copy_(dout[b], non_blocking=True)
            y_free[b].record(cout)
        join_in.record(cin)
        join_out.record(cout)
        comp.wait_event(join_in)
        comp.wait_event(join_out)

    run(min(steps, 2 * G))  # warm the host-side caches outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=comp):
        run(steps)
    with torch.cuda.stream(comp):
        for _ in range(max(1, warmup // steps + 1)):
            graph.replay()
    times = []
    for r in range(repeats):
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        with torch.cuda.stream(comp):
            graph.replay()
        e1.record(comp)
        torch.cuda.synchronize()
        barrier(world)
        times.append(max_over_ranks(e0.elapsed_time(e1), world))
    del graph
    return statistics.median(times), T * H * 4, T * H * 4


def algorithmic_bytes(ls, unique, pairs):
    """Bytes the layer must move at minimum (weights of the experts hit once,
    router weights, activations in and out, routing outputs)."""
    wtype, H, I, E, K, T = ls.wtype, ls.H, ls.I, ls.E, ls.K, ls.T
    bb = 18 if wtype == 2 else 34
    gu_e = 2 * I * (H // 32) * bb
    dn_e = H * (I // 32) * bb
    router = E * H * 4 if ls.routing == "router" else T * E * 4
    layer = unique * (gu_e + dn_e) + router + T * H * 4 * 2 + T * E * 4 + T * K * 8
    gate_up = unique * gu_e + T * H + T * (H // 32) * 8 + pairs * I * 4
    return layer, gate_up


def nvlink_record(ls, step_ms, kern, n, world):
    """The exchange's NVLink figures for one rank (the maximum over ranks of
    the bytes received): bytes per step, the time the step spends outside
    the library's expert kernels, and the peer-copy roofline of those bytes."""
    nv = int(max_over_ranks(float(ls.nvlink_bytes()), world))
    exch = [k for k in kern if k.startswith("ep_")]
    rec = {"bytes_received_per_rank_per_step": nv, "peer_copy_peak_GBs": 770.0,
           "roofline_ms_per_step": round(nv / 770e9 * 1e3, 5), "exchange": ls.ep.exchange}
    if exch:
        rec["exchange_kernels_ms_per_step"] = {k: round(kern[k] / n, 5) for k in exch}
    else:
        rec["ms_outside_library_kernels_per_step"] = round(step_ms - sum(kern.values()) / n, 5)
    return rec


def tensor_roofline(ls, pairs, step_ms, kern, n):
    """Prefill against the dense int8 tensor peak: the expert products' int8
    operations per step (and gate/up's per launch) over their time."""
    peak, src = int8_peak_tops()
    ops, gu_ops = int8_ops(ls, pairs)
    prod_ms = (kern["gate_up"] + kern["down"]) / n
    gu_ms = kern["gate_up"] / n
    return {"bound": "tensor", "unit": "TOPS", "peak": round(peak, 1), "peak_source": src,
            "int8_ops_per_step": ops,
            "layer_achieved": round(ops / (step_ms / 1e3) / 1e12, 2),
            "layer_frac": round(ops / (step_ms / 1e3) / 1e12 / peak, 4),
            "products_achieved": round(ops / (prod_ms / 1e3) / 1e12, 2),
            "products_frac": round(ops / (prod_ms / 1e3) / 1e12 / peak, 4),
            "gate_up_frac": round(gu_ops / (gu_ms / 1e3) / 1e12 / peak, 4),
            "instruction": "mma.sync m16n8k32 (warp-level; the legacy tensor path, not tcgen05)"}


def cpu_baseline(oracle, ls, budget_s=10.0):
    """The reference's CPU algorithm (oracle port) on a bounded sample of the
    workload: the tokens of the bench's inputs in order, one token at a time
    like forward_token, all host threads, for about `budget_s` seconds."""
    wtype, H, I, E, K, T = ls.wtype, ls.H, ls.I, ls.E, ls.K, ls.T
    gu, dn, W = ls.layers[0]
    gu_h, dn_h, W_h = gu.cpu().numpy(), dn.cpu().numpy(), W.cpu().numpy()
    xs = [x.cpu().numpy() for x in ls.xs]
    lgs = [l.cpu().numpy() for l in ls.logit_in] if ls.routing != "router" else None
    threads = os.cpu_count() or 1
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        j, t = divmod(done % (len(xs) * T), T)
        xt = xs[j][t:t + 1]
        if ls.routing == "router":
            _, ids, probs = oracle.router(W_h, xt, H, E, K, 1)
        else:
            ids, probs = oracle.route_from_logits(lgs[j][t:t + 1], E, K, 1)
        oracle.experts(wtype, gu_h, dn_h, ids, probs, None, xt, H, I, E, K, 1, threads)
        done += 1
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{done} tokens, cycling over the bench's {len(xs)} input batches of {T}, one token at a time "
                      f"(model.rs forward_token order), {dt:.1f} s"}


def run_ours(args):
    import torch

    rank, world, local = dist_setup(args.gpus)
    moe, synth = package()
    device = torch.device("cuda", local)
    moe.load_library()
    if args.expert_path:
        moe.set_expert_path(args.expert_path)
    moe.set_speculative_routing(args.spec == 1)
    SPEC["on"] = args.spec == 1
    steps, warmup = args.steps, args.warmup
    hbm_peak, peak_kind = peaks()

    packed = args.weights == "packed"
    if world > 1:
        ls = EPLayerSet(moe, synth, device, args.workload, 8, rank, world, exchange=args.ep_exchange, packed=packed)
    else:
        ls = LayerSet(moe, synth, device, args.workload, n_inputs=8, seed=rank, packed=args.weights == "packed")
    unique, pairs = ls.unique_experts(0)
    graphs = [ls.capture(g) for g in range(2 * ls.n_layers)]
    reps = args.repeats if args.repeats > 0 else repeats_for(ls, steps, warmup, world, graphs)
    rep_stats = {}
    with ClockSampler(local) as clk:
        ms = time_steps(ls, steps, warmup, world, graphs, reps, rep_stats)
    del graphs
    kern = time_kernels(ls, steps)
    e2e_ms, h2d, d2h = time_e2e(ls, steps, warmup, world)
    parity = parity_check(ls, world, rank)

    T = ls.T
    value = world * T * steps / (ms / 1e3)
    strong = args.workload in STRONG
    layer_bytes, gate_up_bytes = algorithmic_bytes(ls, unique, pairs)
    gu_ms = kern["gate_up"] / steps
    top = max(kern, key=kern.get)
    total_kern = sum(kern.values())
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms / steps, 5),
        "timing": {"region": f"{steps} steps", "repeats": rep_stats["repeats"], "reported": "median",
                   "region_ms_min": rep_stats["ms_min"], "region_ms_max": rep_stats["ms_max"]},
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "q4_0 weights x q8_0 activations, int32 block dots, f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights quantised with the reference's Q4_0 rules, N(0,1) x)",
        "config": {"workload": args.workload, "hidden": ls.H, "experts": ls.E, "top_k": ls.K, "expert_ffn": ls.I,
                   "tokens_per_step": world * T, "home_tokens_per_rank": T,
                   "weights": ("Q4_0" if ls.wtype == 2 else "Q8_0") + (
                       " (repacked at load by mrml_moe_prepare_weights)" if packed else " (GGUF layout)"),
                   "parallelism": (f"ep{world} (experts sharded; " + (
                       "sparse Q8_0 row push and partial return over NVLink peer memory, library kernels"
                       if args.ep_exchange == "p2p" else "NCCL all-gather + reduce-scatter") + ")")
                   if world > 1
                   else "single GPU",
                   "l2": f"inputs larger than L2: steps rotate over {ls.n_layers} layer copies "
                         f"({ls.n_layers * ls.layer_bytes / 1e6:.0f} MB of weights)",
                   "unique_experts_step0": unique},
        "roofline": {"bound": "hbm", "kernel": "gate_up", "achieved": round(gate_up_bytes / (gu_ms / 1e3) / 1e9, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(gate_up_bytes / (gu_ms / 1e3) / 1e9 / hbm_peak, 4),
                     "traffic": traffic_from_profile(f"{args.workload}/{args.weights}") if world == 1 else None,
                     "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": gate_up_bytes, "ms_per_launch": round(gu_ms, 5)},
        "layer_roofline": {"achieved": round(layer_bytes / (ms / steps / 1e3) / 1e9, 1), "peak": hbm_peak,
                           "unit": "GB/s", "frac": round(layer_bytes / (ms / steps / 1e3) / 1e9 / hbm_peak, 4),
                           "algorithmic_bytes_per_step": layer_bytes},
        "kernel_share": {k: round(v / total_kern, 4) for k, v in kern.items()},
        "kernel_ms_per_step": {k: round(v / steps, 5) for k, v in kern.items()},
        "top_kernel": top,
        "e2e": {"value": round(world * T * steps / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        # The library's kernels per step, plus the peer exchange's four
        # (push, gather, push, reduce) when the layer runs expert-parallel.
        "gpu_launches": (ls.n_kernels() + (4 if world > 1 and args.ep_exchange == "p2p" else 0)) * steps,
        "clocks": clk.summary(),
    }
    if T >= 2048 and world == 1:
        line["tensor_roofline"] = tensor_roofline(ls, pairs, ms / steps, kern, steps)
    if rank == 0:
        line["parity"] = parity
    if world > 1:
        line["nvlink"] = nvlink_record(ls, ms / steps, kern, steps, world)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
        line["cpu_baseline"] = cpu_baseline(oracle, ls)
    if not args.no_also:
        also = {}
        # (workload, weights packed?): the GGUF-layout headline shape is kept
        # for comparison with the drop-in default layout
        names = ((("c2_t1", packed), ("c2_t8", packed), ("c3_prefill", packed), ("c2_t64", not packed))
                 if world == 1 else ()) + (("c4", packed), ("c4_q8", packed))
        for name, pk in names:
            key = name if pk == packed else name + ("_packed" if pk else "_gguf")
            if name == args.workload and pk == packed:
                continue
            if world > 1:
                ls.close()
            del ls
            gc.collect()
            torch.cuda.empty_cache()
            if world > 1:
                ls = EPLayerSet(moe, synth, device, name, 8, rank, world, exchange=args.ep_exchange, packed=pk)
            else:
                ls = LayerSet(moe, synth, device, name, n_inputs=8, seed=rank, packed=pk)
            u, p = ls.unique_experts(0)
            n = max(steps, 20)
            gr = [ls.capture(g) for g in range(2 * ls.n_layers)]
            m = time_steps(ls, n, max(warmup, 3), world, gr, repeats=3)
            del gr
            k = time_kernels(ls, n)
            lb, gb = algorithmic_bytes(ls, u, p)
            gb_max = max_over_ranks(gb / (k["gate_up"] / n / 1e3) / 1e9 / hbm_peak, world)
            rec = {"tokens_per_s": round(world * ls.T * n / (m / 1e3), 1), "ms_per_step": round(m / n, 5),
                   "tokens_per_step": world * ls.T,
                   "scaling": "strong" if name in STRONG else "weak",
                   "weights": ("Q4_0" if ls.wtype == 2 else "Q8_0") + (" packed" if pk else " GGUF layout"),
                   "layer_hbm_frac": round(lb / (m / n / 1e3) / 1e9 / hbm_peak, 4),
                   "gate_up_hbm_frac": round(gb_max, 4),
                   "kernel_ms_per_step": {kk: round(v / n, 5) for kk, v in k.items()},
                   "unique_experts_step0": u}
            if ls.T * world >= 2048:
                rec["tensor_roofline"] = tensor_roofline(ls, p, m / n, k, n)
            if world > 1:
                rec["nvlink"] = nvlink_record(ls, m / n, k, n, world)
            if name in ("c4", "c4_q8"):
                par = parity_check(ls, world, rank)
                if rank == 0:
                    rec["parity"] = par
            also[key] = rec
        line["also"] = also
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        gc.collect()  # graphs first: they hold the exchange's launches
        torch.cuda.synchronize()
        ls.close()
        dist.destroy_process_group()


def traffic_from_profile(workload, kernel="gate_up"):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    summaries under profiles/ (a line "traffic: <workload>/<weights layout>
    <kernel> <bytes>"), or None."""
    d = os.path.join(ROOT, "profiles")
    try:
        for name in sorted(os.listdir(d)):
            if not name.endswith(".md"):
                continue
            with open(os.path.join(d, name)) as f:
                for line in f:
                    parts = line.split()
                    if len(parts) == 4 and parts[0] == "traffic:" and parts[1] == workload and parts[2] == kernel:
                        return int(parts[3])
    except OSError:
        pass
    return None


def run_reference(args):
    """The reference's CPU MoE path (the C restatement under oracle/; the
    reference's Rust cannot be built here) on the host cores, for the same
    workload as our arm.  Nothing here touches the GPU or this library: inputs
    are generated on the host (numpy streams; expert weights quantised with
    the oracle's C quantisers, the reference's rules).  A step is the whole
    T-token batch: the router over the batch, then the experts one token at a
    time as forward_token runs them (model.rs:2111-2165), row-parallel GEMVs
    on every host thread.  For config 5 a step is one token through the
    30-layer stack (one layer's weights reused), a bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    synth = _load("mrml_moe_b200_synth", os.path.join(ROOT, "qt_llama.cpp_b200", "synth.py"))
    oracle = _load("mrml_oracle", os.path.join(ROOT, "oracle", "oracle.py"))
    stack = args.workload == "c5"
    wtype, H, I, E, K, T, routing = WORKLOADS["c2_t64" if stack else args.workload]
    if args.workload in STRONG:
        T = 64  # config 4's 8192-token step is sampled as 64-token batches on the host
    t_setup = time.perf_counter()
    gu, dn = synth.expert_weights(1, wtype, H, I, E, quantize_fn=oracle.quantize)
    W = synth.normal(1000, E * H, 0.02).reshape(E, H)
    n_batches = 4
    xs = [synth.normal(77 + j, T * H).reshape(T, H) for j in range(n_batches)]
    bias = synth.zipf_bias(5, E)
    lgs = [(synth.normal(900 + j, T * E).reshape(T, E) + bias[None, :]).astype(np.float32) for j in range(n_batches)]
    setup_s = time.perf_counter() - t_setup
    threads = os.cpu_count() or 1

    nw = [(1.0 + synth.normal(1100 + j, H, 0.1)).astype(np.float32) for j in range(4)]

    def one_stack(i):
        h = xs[0][i % 32:i % 32 + 1]
        for _ in range(StackSet.N_LAYERS):
            _, _, xm, rx = oracle.ffn_prologue(h, None, None, None, nw[0], nw[1])
            _, ids, probs = oracle.router(W, rx, H, E, K, 1)
            y = oracle.experts(wtype, gu, dn, ids, probs, None, xm, H, I, E, K, 1, threads)
            h = oracle.ffn_epilogue(h, None, y, None, nw[2], nw[3], 1.0)
        return 1

    def one(i):
        if stack:
            return one_stack(i)
        x = xs[i % n_batches]
        if routing == "router":
            _, ids, probs = oracle.router(W, x, H, E, K, T)
        else:
            ids, probs = oracle.route_from_logits(lgs[i % n_batches], E, K, T)
        for t in range(T):  # forward_token processes one token at a time
            oracle.experts(wtype, gu, dn, ids[t:t + 1], probs[t:t + 1], None, x[t:t + 1], H, I, E, K, 1, threads)
        return T

    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    tokens = sum(one(args.warmup + i) for i in range(args.steps))
    dt = time.perf_counter() - t0
    v = tokens / dt
    per_step = 1 if stack else T
    sample = (f"1 token through the {StackSet.N_LAYERS}-layer stack (one layer's weights reused) per step" if stack
              else f"the whole {T}-token batch per step ({args.steps} steps, {tokens} tokens, {dt:.1f} s), "
                   "one token at a time through the experts")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 3), "unit": "tokens/s", "higher_is_better": True, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "scaling": "strong" if args.workload in STRONG else "weak", "vs_baseline": None,
        "dtype": "q4_0 weights x q8_0 activations, int32 block dots, f32 accumulate" if wtype == 2 else
                 "q8_0 weights x q8_0 activations, int32 block dots, f32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights quantised with the reference's rules, N(0,1) x), host-generated",
        "config": {"workload": args.workload, "hidden": H, "experts": E, "top_k": K, "expert_ffn": I,
                   "tokens_per_step": per_step, "weights": "Q4_0" if wtype == 2 else "Q8_0",
                   "parallelism": "host CPU, row-parallel GEMVs"},
        "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": round(setup_s, 1),
        "note": "reference is Rust (no toolchain here); the oracle/ C restatement of its CPU MoE path is timed",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2_t64", choices=sorted(WORKLOADS) + ["c5"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-also", action="store_true")
    ap.add_argument("--weights", default="packed", choices=["gguf", "packed"],
                    help="expert weights as the GGUF slabs (the reference's layout) or repacked at load time by "
                         "mrml_moe_prepare_weights")
    ap.add_argument("--repeats", type=int, default=0,
                    help="repeats of the timed K-step region (median reported); 0 = enough for ~0.3 s")
    ap.add_argument("--ep-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel exchange for --gpus N > 1")
    ap.add_argument("--expert-path", type=int, default=0,
                    help="MRML_OPTION_EXPERT_PATH: 0 automatic, 1 decode dp4a, 2 tcgen05, 3 general, 4 decode MMA")
    ap.add_argument("--spec", type=int, default=0, choices=[0, 1],
                    help="MRML_OPTION_SPECULATIVE_ROUTING: speculative routing up to 32 tokens (1) or the "
                         "router on the critical path (0, the library's default)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c5":
        run_stack(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
