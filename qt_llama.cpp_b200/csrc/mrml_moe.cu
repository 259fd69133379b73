// mrml_moe.cu — the C ABI of libmrml_moe_b200.so (declared in
// include/mrml_moe.h): argument checks, the workspace layout and the order
// of kernel launches on the caller's stream.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <stdint.h>
#include <stdio.h>

#include "../../include/mrml_moe.h"
#include "checks.h"
#include "common.cuh"
#include "kernels.h"

namespace {

using mrml::kQ4_0;
using mrml::kQ8_0;

using mrml::check_router_args;
constexpr int kMaxE = mrml::kMaxExperts;
constexpr int kMaxK = mrml::kMaxTopK;

// Optional per-launch profiling events (thread-local; see
// mrml_moe_profile_events).  Slot 2i is recorded before launch i of a call,
// slot 2i+1 after it.
thread_local cudaEvent_t* t_events = nullptr;
thread_local int t_n_events = 0;
thread_local int t_next_event = 0;

// Records an event on `s`; under stream capture it becomes an event-record
// node of the graph (cudaEventRecordExternal), so it can be timed on replay.
void record_event(cudaEvent_t e, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
  else
    cudaEventRecord(e, s);
}

struct LaunchMark {
  cudaStream_t s;
  explicit LaunchMark(cudaStream_t st) : s(st) {
    if (t_events && t_next_event + 1 < t_n_events) record_event(t_events[t_next_event], s);
  }
  ~LaunchMark() {
    if (t_events && t_next_event + 1 < t_n_events) {
      record_event(t_events[t_next_event + 1], s);
      t_next_event += 2;
    }
  }
};

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Largest token tile of the tensor-core path; position buffers carry this
// much slack so that a tile starting at the last position stays in bounds.
constexpr int kMaxNT = 64;
// Batches from which the decode kernel's operand is quantised per token and
// then gathered per position group (see run_experts).
constexpr int kGatherMinTokens = 256;

// Positions after padding every expert's segment to a multiple of 16.
int npad_alloc(int E, int K, int T) { return (((T * K + 16 * E) + 15) & ~15) + kMaxNT; }

// Work units of one product: sum over experts of ceil(c_e / NT) row-tile
// columns, at most T*K/NT (rounded up) plus one partial tile per expert that
// has pairs, of which there are at most min(E, T*K).
int units_bound(int E, int K, int T, int NT, int rows, int rows_per_unit) {
  return ((T * K + NT - 1) / NT + std::min(E, T * K)) * ((rows + rows_per_unit - 1) / rows_per_unit);
}

// Workspace regions (each 256-byte aligned), in order.  Positions are the
// padded, expert-grouped order produced by the dispatch kernel.
struct Workspace {
  int* status;       // [0] device status word, [1] reserved (0), [2..3] unit counts
  int8_t* xq;        // [T][H]        Q8_0 values of the layer input (CUDA-core path)
  float* xd;         // [T][H/32]     decoded Q8_0 scales
  int32_t* xsum;     // [T][H/32]     sums of the Q8_0 values per block
  int32_t* cnt;      // [E]           pairs per expert
  int32_t* poff;     // [E+1]         padded segment start per expert
  int32_t* pair_at;  // [npad]        pair at each position (-1 padding)
  int32_t* pos;      // [T*K]         position of each pair (-1 skipped)
  int4* units_gu;    // tensor-core work units, gate/up
  int4* units_dn;    // tensor-core work units, down
  int8_t* xb;        // [H/32][npad/8][256]  tensor-core B operand of gate/up
  int2* xs;          // its scales: [H/32][npad] int2, or group-major records (decode kernel)
  int8_t* ab;        // [I/32][npad/8][256]  B operand of down (re-quantised act)
  int2* as;          // its scales, laid out as xs
  int32_t* chunk_cnt;  // [T*K/1024][E] per-chunk expert counts of the large-batch dispatch
  float* act;        // [npad][I]     geglu output per position (CUDA-core path)
  float* ydown;      // [npad][H]     down output per position (unscaled)
  // Speculative routing (T <= kDispatchTopkMaxTokens): pair arrays above hold
  // T * C candidate slots instead of T * K.
  float* lo;         // [T][E]        router logit intervals
  float* hi;
  int32_t* cand;     // [T][C]        candidate experts per token
  float* cand_w;     // [T][C]        1 for a candidate, 0 for an unused slot
  int npad, max_units_gu, max_units_dn;
  size_t bytes;
};

// Pair slots per token the workspace holds: the speculative path's C
// candidates for small batches, else K.
int pair_slots(int E, int K, int T) {
  return T <= mrml::kDispatchTopkMaxTokens ? std::max(K, mrml::spec_slots(E, K)) : K;
}

Workspace carve(void* base, int H, int I, int E, int K, int T) {
  Workspace w;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(n);
    return r;
  };
  const int Ks = pair_slots(E, K, T);
  const size_t nb = (size_t)H / 32, nbi = (size_t)I / 32, tk = (size_t)T * Ks;
  const int npad = npad_alloc(E, Ks, T);
  w.npad = npad;
  w.max_units_gu = units_bound(E, Ks, T, mrml::kGvTokens, I, mrml::kGvRowsGateUp);
  w.max_units_dn = units_bound(E, Ks, T, mrml::kGvTokens, H, 128);
  w.status = reinterpret_cast<int*>(take(256));
  w.xq = reinterpret_cast<int8_t*>(take((size_t)T * H));
  w.xd = reinterpret_cast<float*>(take((size_t)T * nb * 4));
  w.xsum = reinterpret_cast<int32_t*>(take((size_t)T * nb * 4));
  w.cnt = reinterpret_cast<int32_t*>(take((size_t)E * 4));
  w.poff = reinterpret_cast<int32_t*>(take((size_t)(E + 1) * 4));
  w.pair_at = reinterpret_cast<int32_t*>(take((size_t)npad * 4));
  w.pos = reinterpret_cast<int32_t*>(take(tk * 4));
  w.units_gu = reinterpret_cast<int4*>(take((size_t)w.max_units_gu * 16));
  w.units_dn = reinterpret_cast<int4*>(take((size_t)w.max_units_dn * 16));
  w.xb = reinterpret_cast<int8_t*>(take(nb * npad * 32));
  // int2 per position (tensor cores), or the decode kernel's group-major
  // records (kActScaleBytes per 8 positions)
  const size_t rec_pos = std::max<size_t>(8, mrml::kActScaleBytes / 8);
  w.xs = reinterpret_cast<int2*>(take(nb * npad * rec_pos));
  w.ab = reinterpret_cast<int8_t*>(take(nbi * npad * 32));
  w.as = reinterpret_cast<int2*>(take(nbi * npad * rec_pos));
  w.chunk_cnt = reinterpret_cast<int32_t*>(take(mrml::dispatch_chunk_ints(tk, E) * 4));
  w.act = reinterpret_cast<float*>(take((size_t)npad * I * 4));
  w.ydown = reinterpret_cast<float*>(take((size_t)npad * H * 4));
  const size_t te = T <= mrml::kDispatchTopkMaxTokens ? (size_t)T * E : 0;
  w.lo = reinterpret_cast<float*>(take(te * 4));
  w.hi = reinterpret_cast<float*>(take(te * 4));
  w.cand = reinterpret_cast<int32_t*>(take(te ? tk * 4 : 0));
  w.cand_w = reinterpret_cast<float*>(take(te ? tk * 4 : 0));
  w.bytes = off;
  return w;
}

// Expert-product path (MRML_OPTION_EXPERT_PATH): 0 = automatic, else the
// forced path; process-wide, set from any host thread.
std::atomic<int> g_path{0};

// Bytes of expert gate/up weights the router kernel asks the L2 for
// (MRML_OPTION_L2_PREFETCH_MIB; 0 off).
std::atomic<long long> g_prefetch_bytes{64ll << 20};

// Speculative routing of small batches (MRML_OPTION_SPECULATIVE_ROUTING):
// 0 off (default), 1 on.  Measured on B200 at config 2 it saved the router's
// chain on the critical path (13.0 us serialised against the intervals'
// 6.7 us at T = 1) but the join of the side stream before the combine cost
// about as much: 44.8 against 45.2 us per layer step at T = 1, 81.4 against
// 78.4 us at T = 8, equal at config 5.
std::atomic<int> g_spec{0};

// A library-owned stream per device on which the exact router of the
// speculative path runs beside the expert products, with its fork and join
// events.  Created on first use and kept for the life of the process; the
// mutex keeps one call's fork ... join sequence whole when host threads share
// a device.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool failed = false;
  std::mutex mu;
};
SideStream g_side[mrml::kMaxDevices];
std::mutex g_side_init;

SideStream* side_stream() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= mrml::kMaxDevices) return nullptr;
  SideStream& ss = g_side[dev];
  std::lock_guard<std::mutex> lk(g_side_init);
  if (ss.s || ss.failed) return ss.s ? &ss : nullptr;
  // Creating a stream is not allowed while a capture in the global mode is
  // under way; the relaxed mode lets this thread do it.
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  cudaStream_t st = nullptr;
  cudaEvent_t f = nullptr, j = nullptr;
  const bool ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&f, cudaEventDisableTiming) == cudaSuccess &&
                  cudaEventCreateWithFlags(&j, cudaEventDisableTiming) == cudaSuccess;
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (!ok) {
    (void)cudaGetLastError();
    ss.failed = true;
    return nullptr;
  }
  ss.s = st;
  ss.fork = f;
  ss.join = j;
  return &ss;
}

// Once per device: is it an sm_100 part?
int check_device() {
  static std::atomic<int> verdict[mrml::kMaxDevices];  // 0 unknown, 1 ok, -1 wrong arch
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MRML_ERR_CUDA;
  int v = dev >= 0 && dev < mrml::kMaxDevices ? verdict[dev].load(std::memory_order_relaxed) : 0;
  if (v == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return MRML_ERR_CUDA;
    v = major == 10 ? 1 : -1;
    if (dev >= 0 && dev < mrml::kMaxDevices) verdict[dev].store(v, std::memory_order_relaxed);
  }
  return v == 1 ? MRML_OK : MRML_ERR_DEVICE;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? MRML_OK : MRML_ERR_CUDA; }

#define MRML_TRY(expr)                 \
  do {                                 \
    const int _st = (expr);            \
    if (_st != MRML_OK) return _st;    \
  } while (0)

// Weight type without the packed-layout flag, and the flag.
int base_type(int wtype) { return wtype & ~MRML_PACKED; }
bool is_packed(int wtype) { return (wtype & MRML_PACKED) != 0; }

// Weight type and the shapes it constrains (E experts' slabs).
int check_weights(int wtype, int H, int I, int E, int K, int T) {
  const int wt = base_type(wtype);
  if (wt != MRML_Q4_0 && wt != MRML_Q8_0) return MRML_ERR_UNSUPPORTED;
  if ((wtype & ~(MRML_PACKED | 0xff)) != 0) return MRML_ERR_UNSUPPORTED;
  if (is_packed(wtype) && (H <= 0 || I <= 0 || H % 32 != 0 || I % 32 != 0 || !mrml::gv_packed_supported(wt, H, I)))
    return MRML_ERR_UNSUPPORTED;
  if (H <= 0 || I <= 0 || E <= 0 || K <= 0 || T < 0 || K > E) return MRML_ERR_INVALID_ARGUMENT;
  if (H % 32 != 0 || I % 32 != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (E > kMaxE || K > kMaxK) return MRML_ERR_UNSUPPORTED;
  if ((long long)T * K > (1ll << 30)) return MRML_ERR_UNSUPPORTED;
  if (mrml::gate_up_tok_chunk(wt, H) == 0 || mrml::down_tok_chunk(wt, I) == 0) return MRML_ERR_UNSUPPORTED;
  return MRML_OK;
}

int check_expert_args(int wtype, const uint8_t* gate_up, const uint8_t* down, const int32_t* ids, const float* probs,
                      const float* x, const float* out, int H, int I, int E, int K, int T) {
  MRML_TRY(check_weights(wtype, H, I, E, K, T));
  if (T > 0 && (!gate_up || !down || !ids || !probs || !x || !out)) return MRML_ERR_INVALID_ARGUMENT;
  if (T > 0 && (!aligned16(gate_up) || !aligned16(down) || !aligned16(x))) return MRML_ERR_INVALID_ARGUMENT;
  return MRML_OK;
}

int check_workspace(void* ws, size_t ws_bytes, int H, int I, int E, int K, int T) {
  if (!ws) return MRML_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)ws & 255u) != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (ws_bytes < carve(nullptr, H, I, E, K, T).bytes) return MRML_ERR_WORKSPACE_TOO_SMALL;
  return MRML_OK;
}

#define MRML_LAUNCH(expr)              \
  do {                                 \
    LaunchMark _mark(s);               \
    MRML_TRY(cuda_status(expr));       \
  } while (0)

// The L2 prefetch of mrml_moe_forward: the first experts' gate/up slabs
// (the decode kernel's first wave of work units reads the experts in id
// order), when the batch is likely to hit nearly every expert (T*K >= 2E:
// 86 % of them or more) and the router launch is the decode-size kernel that
// carries it.  Measured on B200 at config 2: T = 64 0.1410 -> 0.1390 ms,
// T = 32 neutral, T = 16 (T*K = E, 63 % hit) 0.1013 -> 0.1065 ms, a loss.
size_t prefetch_bytes(int wtype, int H, int I, int E, int K, int T) {
  if ((long long)T * K < 2ll * E || T > 256) return 0;
  const size_t slab = (size_t)E * 2 * I * (H / 32) * mrml::block_bytes(base_type(wtype));
  const size_t want = (size_t)g_prefetch_bytes.load(std::memory_order_relaxed);
  return std::min(slab, want) & ~(size_t)15;
}

int run_router(const Workspace& w, const float* W, const float* x, float* logits, int32_t* ids, float* probs, int H,
               int E, int K, int T, cudaStream_t s, const uint8_t* prefetch = nullptr, size_t prefetch_bytes = 0) {
  MRML_LAUNCH(mrml::launch_router_logits(W, x, logits, H, E, T, w.status, s, prefetch, prefetch_bytes));
  MRML_LAUNCH(mrml::launch_router_topk(logits, ids, probs, E, K, T, s));
  return MRML_OK;
}

// Expert-product kernels.  The tensor cores pay off once experts see many
// tokens (prefill); at decode sizes one MMA per quant block wastes most of
// each MMA, and the pipelined dp4a kernel is faster.  Shapes outside both
// kernels' limits (H not a multiple of 256) use the general dp4a kernels.
enum Route { kRouteGeneral = 0, kRouteGemv = 1, kRouteTensor = 2, kRouteGemvMma = 3 };

// `pairs` is the expected number of (token, slot) pairs this call computes:
// T * K on one device, about T * K * E / e_total for an expert shard.
Route pick_route(int wtype, bool packed, int H, int I, int E, long long pairs) {
  const bool tc = mrml::tc_supported(wtype, H, I, 64) && mrml::tc_supported(wtype, H, I, 16);
  const bool gv = mrml::gv_supported(wtype, H, I);
  const int forced = g_path.load(std::memory_order_relaxed);
  // Packed weights run on the decode kernel only (its MMA or dp4a form).
  // The MMA form from a quarter of a pair per expert: measured on B200 at
  // config 2, T = 8 (half a pair per expert) it takes the layer step from
  // 93 to 81 us; at T = 1 the dp4a form is faster (45 vs 49 us).
  const bool mma_size = pairs * 4 >= E;
  if (packed) return forced == 1 ? kRouteGemv : forced == 4 || mma_size ? kRouteGemvMma : kRouteGemv;
  switch (forced) {
    case 1: return gv ? kRouteGemv : kRouteGeneral;
    case 2: return tc ? kRouteTensor : (gv ? kRouteGemv : kRouteGeneral);
    case 3: return kRouteGeneral;
    case 4: return gv ? kRouteGemvMma : kRouteGeneral;
    default: break;
  }
  if (!gv) return tc && pairs > 16ll * E ? kRouteTensor : kRouteGeneral;
  // A warp-level MMA covers 8 positions whatever the count; it also beats the tcgen05 kernel
  // at every measured prefill size (config 3: 123 vs 169 us gate/up; the C2
  // layer at 2048 tokens, Q8_0: 1.40 vs 2.48 ms), because the exact f32
  // rescale per quant block, not the integer products, bounds both, and the
  // warp-level MMA leaves its sums in registers.
  return mma_size ? kRouteGemvMma : kRouteGemv;
}

// CTAs per SM of the decode kernel's two products (0: its automatic
// choice), from the expected work units per SM: the experts hit, about
// E (1 - exp(-pairs / E)), times the row tiles of each.  Measured on B200 at
// config 2 (packed Q4_0, warp MMA, units of 8 positions): 3 CTAs with deeper
// rings for the down product from about 10 units per SM (T = 16, 32 and 64:
// 0.1387 -> 0.1327 ms at T = 64) but not at T = 8 (7.5 per SM), and for
// gate/up between 4.5 and 7.5 units per SM (T = 16: 0.1120 -> 0.1059 ms; the
// expert shard of 2-GPU expert parallelism, 4.8 per SM: 0.1625 -> 0.1600 ms),
// where the 5 of the automatic choice lost; elsewhere the automatic choice.
void decode_ctas_per_sm(int wtype, bool packed, bool mma, int ng_gu, int ng_dn, int E, long long pairs, int mt_gu,
                        int mt_dn, int& per_gu, int& per_dn) {
  per_gu = per_dn = 0;
  if (!packed || !mma || wtype != MRML_Q4_0 || E <= 0) return;
  const double hit = E * (1.0 - std::exp(-(double)pairs / E));
  const double sms = (double)mrml::tc_num_sms();
  const double u_gu = hit * mt_gu / sms, u_dn = hit * mt_dn / sms;
  if (ng_gu == 1 && u_gu > 4.5 && u_gu <= 7.5) per_gu = 3;
  if (ng_dn == 1 && u_dn > 10.0) per_dn = 3;
}

// With topk_logits, the dispatch kernel first selects the experts from the
// router logits and writes ids/probs (ids_out/probs_out, the buffers that
// ids/probs point to), replacing the top-k launch (small batches).
//
// With spec (small batches), the dispatch selects candidate experts from the
// router logits' intervals into the workspace's C slots per token (the pair
// arrays then hold T * C slots); the products run over the candidates, and
// the combine, after the stream waits on `join` (the exact router's ids and
// probs are then ready), takes the reference's K slots from ids / probs.
int run_experts(const Workspace& w, int wtype, const uint8_t* gate_up, const uint8_t* down, const int32_t* ids,
                const float* probs, const float* down_scale, const float* x, float* out, int H, int I, int E, int K,
                int T, cudaStream_t s, int e_first = 0, int e_total = 0, const float* topk_logits = nullptr,
                int32_t* ids_out = nullptr, float* probs_out = nullptr, const mrml::SpecRoute* spec = nullptr,
                cudaEvent_t join = nullptr) {
  if (e_total == 0) e_total = E;
  // slots per token of the pair arrays
  const int Kp = spec ? spec->C : K;
  const bool packed = is_packed(wtype);
  wtype = base_type(wtype);
  const long long pairs = (long long)T * K * E / e_total;
  const Route route = pick_route(wtype, packed, H, I, E, pairs);
  const bool gv = route == kRouteGemv || route == kRouteGemvMma;
  // Work units of 16 positions (two groups of 8) on the MMA form once
  // experts see about 12 tokens or more: a weight stage and each unpacked
  // row fragment then serve twice the positions.  Measured on B200: faster
  // for both products with Q4_0 weights and for the Q8_0 down product; the
  // Q8_0 gate/up kernel needs more registers for them (3 CTAs per SM instead
  // of 5) and lost at config 3, so it keeps units of 8.
  const bool two = route == kRouteGemvMma && pairs >= 12ll * E && mrml::gv_two_groups_supported(wtype, H, I);
  const int ng_gu = two && wtype == MRML_Q4_0 ? 2 : 1, ng_dn = two ? 2 : 1;
  const int NT = gv ? mrml::kGvTokens * ng_gu : (pairs > 12ll * E ? 64 : 16);
  const int NT_dn = gv ? mrml::kGvTokens * ng_dn : NT;
  const int rows_gu = gv ? mrml::kGvRowsGateUp : 128;
  const int mt_gu = (I + rows_gu - 1) / rows_gu, mt_dn = (H + 127) / 128;  // down tiles: 128 rows on both paths
  int* n_units = w.status + 2;
  // From kGatherMinTokens tokens the decode kernel's operand is built in two
  // steps: the input quantised once per token (before the dispatch, which it
  // does not depend on), then gathered per position group after it.
  const bool gather = gv && T >= kGatherMinTokens;
  if (gather) MRML_LAUNCH(mrml::launch_quantize_rows(x, w.xq, w.xd, w.xsum, (long long)T * (H / 32), s));
  const int32_t* pids = spec ? w.cand : ids;
  const float* pprobs = spec ? w.cand_w : probs;
  MRML_LAUNCH(mrml::launch_dispatch(pids, pprobs, T * Kp, E, e_first, e_total, w.cnt, w.poff, w.pair_at, w.pos,
                                    w.units_gu, w.units_dn, n_units, NT, NT_dn, mt_gu, rows_gu, mt_dn, w.status, s,
                                    topk_logits, Kp, spec ? w.cand : ids_out, spec ? w.cand_w : probs_out,
                                    w.chunk_cnt, spec));
  if (route == kRouteGeneral) {
    MRML_LAUNCH(mrml::launch_quantize_rows(x, w.xq, w.xd, w.xsum, (long long)T * (H / 32), s));
    MRML_LAUNCH(mrml::launch_gate_up(wtype, gate_up, w.cnt, w.poff, w.pair_at, w.xq, w.xd, w.xsum, w.act, H, I, E, Kp,
                                     w.status, s));
    MRML_LAUNCH(mrml::launch_down(wtype, down, w.cnt, w.poff, w.act, w.ydown, H, I, E, w.status, s));
  } else {
    const int mu_gu = units_bound(E, Kp, T, NT, I, rows_gu), mu_dn = units_bound(E, Kp, T, NT_dn, H, 128);
    if (gather)
      MRML_LAUNCH(mrml::launch_gather_groups(wtype, w.xq, w.xd, w.xsum, w.pair_at, w.poff + E, H, Kp, w.npad, w.xb,
                                             w.xs, s));
    else
      MRML_LAUNCH(mrml::launch_quantize_scatter(wtype, x, w.pos, T, H, Kp, w.npad, gv, w.xb, w.xs, s));
    if (route == kRouteTensor) {
      MRML_LAUNCH(mrml::launch_gemm_tc(0, wtype, NT, gate_up, H, I, E, w.xb, w.xs, w.units_gu, n_units, mu_gu,
                                       w.npad, w.ab, w.as, nullptr, w.status, s));
      MRML_LAUNCH(mrml::launch_gemm_tc(1, wtype, NT, down, H, I, E, w.ab, w.as, w.units_dn, n_units + 1, mu_dn,
                                       w.npad, nullptr, nullptr, w.ydown, w.status, s));
    } else {
      const bool mma = route == kRouteGemvMma;
      int per_gu = 0, per_dn = 0;
      decode_ctas_per_sm(wtype, packed, mma, ng_gu, ng_dn, E, pairs, mt_gu, mt_dn, per_gu, per_dn);
      MRML_LAUNCH(mrml::launch_gemv(0, wtype, packed, mma, ng_gu, gate_up, H, I, E, w.xb, w.xs, w.units_gu, n_units,
                                    mu_gu, w.npad, w.ab, w.as, nullptr, w.status, s, per_gu));
      MRML_LAUNCH(mrml::launch_gemv(1, wtype, packed, mma, ng_dn, down, H, I, E, w.ab, w.as, w.units_dn, n_units + 1,
                                    mu_dn, w.npad, nullptr, nullptr, w.ydown, w.status, s, per_dn));
    }
  }
  if (spec) {
    if (join) MRML_TRY(cuda_status(cudaStreamWaitEvent(s, join, 0)));
    MRML_LAUNCH(mrml::launch_combine_spec(w.ydown, w.pos, w.cand, ids, probs, down_scale, out, H, K, Kp, T, w.status,
                                          s));
    return MRML_OK;
  }
  MRML_LAUNCH(mrml::launch_combine(w.ydown, w.pos, ids, probs, down_scale, out, H, K, T, s));
  return MRML_OK;
}

// The expert-parallel workspace: the shard's expert workspace for N*T
// tokens and E/N experts, then the received ids / weights [N*T][K] and the
// published row pointers of the step (values, f16 scales).
struct EpExtras {
  int32_t* ids_all;
  float* probs_all;
  const uint8_t** rows;
  size_t bytes;
};

EpExtras carve_ep(void* base, int N, int T, int K) {
  EpExtras x;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(n);
    return r;
  };
  x.ids_all = reinterpret_cast<int32_t*>(take((size_t)N * T * K * 4));
  x.probs_all = reinterpret_cast<float*>(take((size_t)N * T * K * 4));
  x.rows = reinterpret_cast<const uint8_t**>(take(2 * sizeof(void*)));
  x.bytes = off;
  return x;
}

size_t ep_workspace_bytes(int N, int T, int H, int I, int E, int K) {
  return carve(nullptr, H, I, E / N, K, N * T).bytes + carve_ep(nullptr, N, T, K).bytes;
}

int check_ep_args(void* const* slabs, int rank, int N, int T, int H, int E, int K) {
  if (!slabs || N < 1 || N > mrml::kEpMaxRanks || rank < 0 || rank >= N || T < 1 || H < 32 || H % 32 != 0 || K < 1)
    return MRML_ERR_INVALID_ARGUMENT;
  if (E < N || E % N != 0 || K > E) return MRML_ERR_INVALID_ARGUMENT;
  if (E > kMaxE || K > kMaxK) return MRML_ERR_UNSUPPORTED;
  return MRML_OK;
}

// The experts of this rank on the tokens every rank sent it (see
// mrml_moe_ep_experts): receive, dispatch over the N*T received tokens'
// pairs on this rank's experts, the group-major operand gathered from the
// received Q8_0 rows, gate/up, down, then the partials pushed home.
int run_ep_experts(void* ws, int wtype, const uint8_t* gate_up, const uint8_t* down, const float* down_scale,
                   uint8_t* const* slabs, int rank, int N, int T, int H, int I, int E, int K, cudaStream_t s) {
  const int Ec = E / N, NT = N * T;
  const Workspace w = carve(ws, H, I, Ec, K, NT);
  const EpExtras x = carve_ep(static_cast<uint8_t*>(ws) + w.bytes, N, T, K);
  const bool packed = is_packed(wtype);
  wtype = base_type(wtype);
  const long long pairs = (long long)T * K;  // expected pairs on this rank
  const Route route = pick_route(wtype, packed, H, I, Ec, pairs);
  if (route != kRouteGemv && route != kRouteGemvMma) return MRML_ERR_UNSUPPORTED;
  const bool two = route == kRouteGemvMma && pairs >= 12ll * Ec && mrml::gv_two_groups_supported(wtype, H, I);
  const int ng_gu = two && wtype == MRML_Q4_0 ? 2 : 1, ng_dn = two ? 2 : 1;
  const int NT_gu = mrml::kGvTokens * ng_gu, NT_dn = mrml::kGvTokens * ng_dn;
  const int rows_gu = mrml::kGvRowsGateUp;
  const int mt_gu = (I + rows_gu - 1) / rows_gu, mt_dn = (H + 127) / 128;
  int* n_units = w.status + 2;
  MRML_LAUNCH(mrml::launch_ep_recv(slabs, rank, N, T, H, K, x.ids_all, x.probs_all, x.rows, w.status, s));
  MRML_LAUNCH(mrml::launch_dispatch(x.ids_all, x.probs_all, NT * K, Ec, rank * Ec, E, w.cnt, w.poff, w.pair_at,
                                    w.pos, w.units_gu, w.units_dn, n_units, NT_gu, NT_dn, mt_gu, rows_gu, mt_dn,
                                    w.status, s, nullptr, 0, nullptr, nullptr, w.chunk_cnt));
  MRML_LAUNCH(mrml::launch_ep_gather(wtype, x.rows, w.pair_at, w.poff + Ec, H, K, w.npad, w.xb, w.xs, s));
  const int mu_gu = units_bound(Ec, K, NT, NT_gu, I, rows_gu), mu_dn = units_bound(Ec, K, NT, NT_dn, H, 128);
  const bool mma = route == kRouteGemvMma;
  int per_gu = 0, per_dn = 0;
  decode_ctas_per_sm(wtype, packed, mma, ng_gu, ng_dn, Ec, pairs, mt_gu, mt_dn, per_gu, per_dn);
  MRML_LAUNCH(mrml::launch_gemv(0, wtype, packed, mma, ng_gu, gate_up, H, I, Ec, w.xb, w.xs, w.units_gu, n_units,
                                mu_gu, w.npad, w.ab, w.as, nullptr, w.status, s, per_gu));
  MRML_LAUNCH(mrml::launch_gemv(1, wtype, packed, mma, ng_dn, down, H, I, Ec, w.ab, w.as, w.units_dn, n_units + 1,
                                mu_dn, w.npad, nullptr, nullptr, w.ydown, w.status, s, per_dn));
  MRML_LAUNCH(mrml::launch_ep_combine_push(slabs, rank, N, T, H, K, w.ydown, w.pos, x.ids_all, x.probs_all,
                                           down_scale, s));
  return MRML_OK;
}

}  // namespace

extern "C" {

int mrml_moe_version(void) { return 100; }

const char* mrml_moe_status_string(int status) {
  switch (status) {
    case MRML_OK: return "ok";
    case MRML_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MRML_ERR_UNSUPPORTED: return "unsupported shape or weight type";
    case MRML_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case MRML_ERR_CUDA: return "CUDA runtime error";
    case MRML_ERR_DEVICE: return "device is not an sm_100 GPU";
    case MRML_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
    case MRML_ERR_BAD_EXPERT_ID: return "expert id out of range";
    case MRML_ERR_NOT_FOUND: return "not found";
    default: return "unknown status";
  }
}

size_t mrml_moe_workspace_bytes(int H, int I, int E, int K, int T) {
  if (H <= 0 || I <= 0 || E <= 0 || K <= 0 || T < 0) return 0;
  return carve(nullptr, H, I, E, K, T).bytes;
}

int mrml_moe_router_logit_bounds(const float* W, const float* x, float* lo, float* hi, int H, int E, int T,
                                 mrml_stream_t stream) {
  if (H <= 0 || E <= 0 || T < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (T > 0 && (!W || !x || !lo || !hi)) return MRML_ERR_INVALID_ARGUMENT;
  if (T == 0) return MRML_OK;
  if (!mrml::router_bounds_supported(W, x, H)) return MRML_ERR_UNSUPPORTED;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_router_bounds(W, x, lo, hi, H, E, T, nullptr, s));
  return MRML_OK;
}

int mrml_moe_router(const float* W, const float* x, float* logits, int32_t* ids, float* probs, int H, int E, int K,
                    int T, void* workspace, size_t workspace_bytes, mrml_stream_t stream) {
  MRML_TRY(check_router_args(W, x, logits, ids, probs, H, E, K, T));
  if (T == 0) return MRML_OK;
  MRML_TRY(check_device());
  // The router itself uses no workspace memory; the size check keeps the
  // documented contract (a workspace of mrml_moe_workspace_bytes for the
  // smallest expert shape).
  MRML_TRY(check_workspace(workspace, workspace_bytes, 32, 32, E, K, T));
  const Workspace w = carve(workspace, 32, 32, E, K, T);
  return run_router(w, W, x, logits, ids, probs, H, E, K, T, (cudaStream_t)stream);
}

int mrml_moe_route_from_logits(const float* logits, int32_t* ids, float* probs, int E, int K, int T,
                               mrml_stream_t stream) {
  if (E <= 0 || K <= 0 || T < 0 || K > E) return MRML_ERR_INVALID_ARGUMENT;
  if (E > kMaxE || K > kMaxK) return MRML_ERR_UNSUPPORTED;
  if (T == 0) return MRML_OK;
  if (!logits || !ids || !probs) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_router_topk(logits, ids, probs, E, K, T, s));
  return MRML_OK;
}

int mrml_moe_experts(int wtype, const uint8_t* gate_up, const uint8_t* down, const int32_t* ids, const float* probs,
                     const float* down_scale, const float* x, float* out, int H, int I, int E, int K, int T,
                     void* workspace, size_t workspace_bytes, mrml_stream_t stream) {
  MRML_TRY(check_expert_args(wtype, gate_up, down, ids, probs, x, out, H, I, E, K, T));
  if (T == 0) return MRML_OK;
  MRML_TRY(check_device());
  MRML_TRY(check_workspace(workspace, workspace_bytes, H, I, E, K, T));
  const Workspace w = carve(workspace, H, I, E, K, T);
  return run_experts(w, wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, K, T, (cudaStream_t)stream);
}

int mrml_moe_experts_shard(int wtype, const uint8_t* gate_up, const uint8_t* down, const int32_t* ids,
                           const float* probs, const float* down_scale, const float* x, float* out, int H, int I,
                           int E, int e_first, int e_count, int K, int T, void* workspace, size_t workspace_bytes,
                           mrml_stream_t stream) {
  if (E <= 0 || e_first < 0 || e_count <= 0 || e_first + e_count > E || E > kMaxE) return MRML_ERR_INVALID_ARGUMENT;
  if (K > E) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_expert_args(wtype, gate_up, down, ids, probs, x, out, H, I, e_count, std::min(K, e_count), T));
  if (T == 0) return MRML_OK;
  MRML_TRY(check_device());
  MRML_TRY(check_workspace(workspace, workspace_bytes, H, I, e_count, K, T));
  const Workspace w = carve(workspace, H, I, e_count, K, T);
  return run_experts(w, wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, e_count, K, T,
                     (cudaStream_t)stream, e_first, E);
}

int mrml_moe_forward(int wtype, const float* router_w, const float* router_x, const float* x, const uint8_t* gate_up,
                     const uint8_t* down, const float* down_scale, float* logits, int32_t* ids, float* probs,
                     float* out, int H, int I, int E, int K, int T, void* workspace, size_t workspace_bytes,
                     mrml_stream_t stream) {
  MRML_TRY(check_router_args(router_w, router_x, logits, ids, probs, H, E, K, T));
  MRML_TRY(check_expert_args(wtype, gate_up, down, ids, probs, x, out, H, I, E, K, T));
  if (T == 0) return MRML_OK;
  MRML_TRY(check_device());
  MRML_TRY(check_workspace(workspace, workspace_bytes, H, I, E, K, T));
  const Workspace w = carve(workspace, H, I, E, K, T);
  const cudaStream_t s = (cudaStream_t)stream;
  // Up to 32 tokens the router's exact sequential chains (H dependent adds,
  // a latency floor) leave the critical path: the logits' intervals, from
  // parallel sums and a rigorous rounding bound, let the dispatch select the
  // candidate experts that can be in the top-K (almost always exactly K);
  // the exact router runs meanwhile on the side stream, and the combine
  // takes its top-K.  Results are those of the plain path, bit for bit.
  if (g_spec.load(std::memory_order_relaxed) && K < E && mrml::dispatch_topk_supported(E, K, T) &&
      mrml::router_bounds_supported(router_w, router_x, H)) {
    SideStream* ss = side_stream();
    if (ss) {
      std::lock_guard<std::mutex> lk(ss->mu);
      const cudaStream_t side = ss->s;
      MRML_TRY(cuda_status(cudaEventRecord(ss->fork, s)));
      MRML_TRY(cuda_status(cudaStreamWaitEvent(side, ss->fork, 0)));
      int st = MRML_OK;
      {
        LaunchMark mark(side);
        st = cuda_status(mrml::launch_router_logits(router_w, router_x, logits, H, E, T, w.status, side));
      }
      if (st == MRML_OK) {
        LaunchMark mark(side);
        st = cuda_status(mrml::launch_router_topk(logits, ids, probs, E, K, T, side));
      }
      // the side stream rejoins the caller's stream on every path
      const int jst = cuda_status(cudaEventRecord(ss->join, side));
      if (st == MRML_OK) st = jst;
      if (st == MRML_OK) {
        LaunchMark mark(s);
        st = cuda_status(mrml::launch_router_bounds(router_w, router_x, w.lo, w.hi, H, E, T, w.status, s));
      }
      const mrml::SpecRoute spec{w.lo, w.hi, router_w, router_x, H, K, mrml::spec_slots(E, K)};
      if (st == MRML_OK)
        st = run_experts(w, wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, K, T, s, 0, 0, nullptr,
                         nullptr, nullptr, &spec, ss->join);
      if (st != MRML_OK && jst == MRML_OK) cudaStreamWaitEvent(s, ss->join, 0);
      return st;
    }
  }
  // Up to 32 tokens the dispatch kernel selects the experts itself (one
  // launch fewer on the decode path); the selection is the same ordering.
  // (At 64 tokens its single CTA took longer than the separate top-k launch.)
  const size_t pf = prefetch_bytes(wtype, H, I, E, K, T);
  if (mrml::dispatch_topk_supported(E, K, T)) {
    MRML_LAUNCH(mrml::launch_router_logits(router_w, router_x, logits, H, E, T, w.status, s, gate_up, pf));
    return run_experts(w, wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, K, T, s, 0, 0, logits, ids,
                       probs);
  }
  MRML_TRY(run_router(w, router_w, router_x, logits, ids, probs, H, E, K, T, s, gate_up, pf));
  return run_experts(w, wtype, gate_up, down, ids, probs, down_scale, x, out, H, I, E, K, T, s);
}

size_t mrml_moe_weights_bytes(int wtype, int H, int I, int E, int which) {
  const int wt = base_type(wtype);
  if ((wt != MRML_Q4_0 && wt != MRML_Q8_0) || H <= 0 || I <= 0 || E <= 0 || H % 32 != 0 || I % 32 != 0) return 0;
  const size_t bb = mrml::block_bytes(wt);
  if (which == 0) return (size_t)E * 2 * I * (H / 32) * bb;
  if (which == 1) return (size_t)E * H * (I / 32) * bb;
  return 0;
}

int mrml_moe_prepare_weights(int wtype, const uint8_t* gate_up, const uint8_t* down, uint8_t* gate_up_packed,
                             uint8_t* down_packed, int H, int I, int E, mrml_stream_t stream) {
  if (wtype != MRML_Q4_0 && wtype != MRML_Q8_0) return MRML_ERR_UNSUPPORTED;
  if (H <= 0 || I <= 0 || E <= 0 || H % 32 != 0 || I % 32 != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (E > kMaxE) return MRML_ERR_UNSUPPORTED;
  if (!gate_up || !down || !gate_up_packed || !down_packed) return MRML_ERR_INVALID_ARGUMENT;
  if (!aligned16(gate_up_packed) || !aligned16(down_packed) || ((uintptr_t)gate_up & 1) || ((uintptr_t)down & 1))
    return MRML_ERR_INVALID_ARGUMENT;
  const size_t gb = mrml_moe_weights_bytes(wtype, H, I, E, 0), db = mrml_moe_weights_bytes(wtype, H, I, E, 1);
  auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return x < y + nb && y < x + na;
  };
  if (overlap(gate_up, gb, gate_up_packed, gb) || overlap(down, db, down_packed, db) ||
      overlap(gate_up_packed, gb, down_packed, db))
    return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  if (!mrml::gv_packed_supported(wtype, H, I)) return MRML_ERR_UNSUPPORTED;
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_TRY(cuda_status(mrml::launch_repack(0, wtype, gate_up, gate_up_packed, H, I, E, s)));
  MRML_TRY(cuda_status(mrml::launch_repack(1, wtype, down, down_packed, H, I, E, s)));
  return MRML_OK;
}

size_t mrml_moe_ep_workspace_bytes(int N, int T, int H, int I, int E, int K) {
  if (N < 1 || T < 1 || H <= 0 || I <= 0 || E < N || E % N != 0 || K <= 0) return 0;
  return ep_workspace_bytes(N, T, H, I, E, K);
}

int mrml_moe_ep_dispatch(void* const* slabs, int rank, int N, int T, int H, int E, int K, const float* x,
                         const int32_t* ids, const float* probs, mrml_stream_t stream) {
  MRML_TRY(check_ep_args(slabs, rank, N, T, H, E, K));
  if (!x || !ids || !probs || !aligned16(x)) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_ep_dispatch(reinterpret_cast<uint8_t* const*>(slabs), rank, N, T, H, E, K, x, ids, probs,
                                       s));
  return MRML_OK;
}

int mrml_moe_ep_experts(int wtype, const uint8_t* gate_up, const uint8_t* down, const float* down_scale,
                        void* const* slabs, int rank, int N, int T, int H, int I, int E, int K, void* workspace,
                        size_t workspace_bytes, mrml_stream_t stream) {
  MRML_TRY(check_ep_args(slabs, rank, N, T, H, E, K));
  MRML_TRY(check_weights(wtype, H, I, E / N, std::min(K, E / N), N * T));
  if (H % 256 != 0 || I % mrml::kGvRowsGateUp != 0) return MRML_ERR_UNSUPPORTED;  // the decode kernel's shapes
  if (!gate_up || !down || !aligned16(gate_up) || !aligned16(down)) return MRML_ERR_INVALID_ARGUMENT;
  if (!workspace || ((uintptr_t)workspace & 255u) != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < ep_workspace_bytes(N, T, H, I, E, K)) return MRML_ERR_WORKSPACE_TOO_SMALL;
  MRML_TRY(check_device());
  return run_ep_experts(workspace, wtype, gate_up, down, down_scale, reinterpret_cast<uint8_t* const*>(slabs), rank,
                        N, T, H, I, E, K, (cudaStream_t)stream);
}

int mrml_moe_ep_combine(void* const* slabs, int rank, int N, int T, int H, int E, int K, const int32_t* ids,
                        const float* probs, float* out, void* workspace, mrml_stream_t stream) {
  MRML_TRY(check_ep_args(slabs, rank, N, T, H, E, K));
  if (!ids || !probs || !out || !workspace || !aligned16(out) || ((uintptr_t)workspace & 255u) != 0)
    return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_ep_reduce(reinterpret_cast<uint8_t* const*>(slabs), rank, N, T, H, E, K, ids, probs, out,
                                     static_cast<int*>(workspace), s));
  return MRML_OK;
}

int mrml_moe_combine(const float* ydown, const int32_t* pos, const int32_t* ids, const float* probs,
                     const float* down_scale, float* out, int H, int K, int T, mrml_stream_t stream) {
  if (H <= 0 || K <= 0 || T < 0 || K > kMaxK) return MRML_ERR_INVALID_ARGUMENT;
  if (T == 0) return MRML_OK;
  if (!ydown || !pos || !ids || !probs || !out) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_combine(ydown, pos, ids, probs, down_scale, out, H, K, T, s));
  return MRML_OK;
}

// model.rs:1730-1784 use eps = 1e-6 for every norm of the FFN block.
constexpr float kFfnEps = 1e-6f;

int mrml_moe_ffn_prologue(const float* hidden, const float* attn, const float* post_attn_norm, const float* ffn_norm,
                          const float* pre_ffw_norm_2, const float* router_scale, float* attn_res, float* shared,
                          float* moe, float* router, int dim, int batch, mrml_stream_t stream) {
  if (dim <= 0 || batch < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (batch == 0) return MRML_OK;
  if (!hidden || (!attn_res && !shared && !moe && !router)) return MRML_ERR_INVALID_ARGUMENT;
  if (mrml::rms_norm_rows_per_cta(dim) == 0) return MRML_ERR_UNSUPPORTED;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_ffn_prologue(hidden, attn, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale,
                                        attn_res, shared, moe, router, dim, batch, kFfnEps, s));
  return MRML_OK;
}

int mrml_moe_ffn_epilogue(const float* attn_res, const float* dense, const float* moe, const float* post_ffw_norm_1,
                          const float* post_ffw_norm_2, const float* post_ffw_norm, float* output, float layer_scale,
                          int dim, int batch, mrml_stream_t stream) {
  if (dim <= 0 || batch < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (batch == 0) return MRML_OK;
  if (!attn_res || !moe || !output) return MRML_ERR_INVALID_ARGUMENT;
  if (mrml::rms_norm_rows_per_cta(2 * dim) == 0) return MRML_ERR_UNSUPPORTED;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_ffn_epilogue(attn_res, dense, moe, post_ffw_norm_1, post_ffw_norm_2, post_ffw_norm,
                                        layer_scale, output, dim, batch, kFfnEps, s));
  return MRML_OK;
}

size_t mrml_moe_dense_ffn_workspace_bytes(int H, int I, int T) {
  if (H <= 0 || I <= 0 || T < 0) return 0;
  return carve(nullptr, H, I, 1, 1, T).bytes + 2 * align256((size_t)T * 4);
}

int mrml_moe_dense_ffn(int wtype, const uint8_t* gate_up, const uint8_t* down, const float* x, float* out, int H,
                       int I, int T, void* workspace, size_t workspace_bytes, mrml_stream_t stream) {
  MRML_TRY(check_weights(wtype, H, I, 1, 1, T));
  if (T == 0) return MRML_OK;
  if (!gate_up || !down || !x || !out || !aligned16(gate_up) || !aligned16(down) || !aligned16(x))
    return MRML_ERR_INVALID_ARGUMENT;
  if (!workspace || ((uintptr_t)workspace & 255u) != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < mrml_moe_dense_ffn_workspace_bytes(H, I, T)) return MRML_ERR_WORKSPACE_TOO_SMALL;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  const Workspace w = carve(workspace, H, I, 1, 1, T);
  int32_t* ids = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + w.bytes);
  float* probs = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + w.bytes + align256((size_t)T * 4));
  MRML_LAUNCH(mrml::launch_dense_routing(ids, probs, T, s));
  return run_experts(w, wtype, gate_up, down, ids, probs, nullptr, x, out, H, I, 1, 1, T, s);
}

// The FFN block's workspace: the expert workspace (its status word first;
// the shared MLP's call reuses the same bytes, one after the other on the
// stream), then the block's activations [T][H] x 6, the router logits and
// the selected ids / weights.
namespace {
struct BlockWs {
  float *attn_res, *shared, *moe_in, *router_in, *mlp_out, *moe_out, *logits, *probs;
  int32_t* ids;
  size_t inner, bytes;
};
BlockWs carve_block(void* base, int H, int I, int I_dense, int E, int K, int T) {
  BlockWs b{};
  b.inner = carve(nullptr, H, I, E, K, T).bytes;
  if (I_dense > 0) b.inner = std::max(b.inner, mrml_moe_dense_ffn_workspace_bytes(H, I_dense, T));
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = align256(b.inner);
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(n);
    return r;
  };
  const size_t row = (size_t)T * H * 4;
  b.attn_res = reinterpret_cast<float*>(take(row));
  b.shared = reinterpret_cast<float*>(take(row));
  b.moe_in = reinterpret_cast<float*>(take(row));
  b.router_in = reinterpret_cast<float*>(take(row));
  b.mlp_out = reinterpret_cast<float*>(take(row));
  b.moe_out = reinterpret_cast<float*>(take(row));
  b.logits = reinterpret_cast<float*>(take((size_t)T * E * 4));
  b.ids = reinterpret_cast<int32_t*>(take((size_t)T * K * 4));
  b.probs = reinterpret_cast<float*>(take((size_t)T * K * 4));
  b.bytes = off;
  return b;
}
}  // namespace

size_t mrml_moe_ffn_block_workspace_bytes(int H, int I, int I_dense, int E, int K, int T) {
  if (H <= 0 || I <= 0 || I_dense < 0 || E <= 0 || K <= 0 || T < 0) return 0;
  return carve_block(nullptr, H, I, I_dense, E, K, T).bytes;
}

int mrml_moe_ffn_block(int wtype, int dense_wtype, float* hidden, const float* attn, const float* post_attn_norm,
                       const float* ffn_norm, const float* pre_ffw_norm_2, const float* router_scale,
                       const float* post_ffw_norm_1, const float* post_ffw_norm_2, const float* post_ffw_norm,
                       float layer_scale, const float* router_w, const uint8_t* gate_up, const uint8_t* down,
                       const float* down_scale, const uint8_t* dense_gate_up, const uint8_t* dense_down, int H, int I,
                       int I_dense, int E, int K, int T, void* workspace, size_t workspace_bytes,
                       mrml_stream_t stream) {
  if (T < 0 || I_dense < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (T == 0) return MRML_OK;
  const bool dense = I_dense > 0;
  if (!hidden || !router_w || (dense && (!dense_gate_up || !dense_down))) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_weights(wtype, H, I, E, K, T));
  if (dense) MRML_TRY(check_weights(dense_wtype, H, I_dense, 1, 1, T));
  if (!workspace || ((uintptr_t)workspace & 255u) != 0) return MRML_ERR_INVALID_ARGUMENT;
  const BlockWs b = carve_block(workspace, H, I, I_dense, E, K, T);
  if (workspace_bytes < b.bytes) return MRML_ERR_WORKSPACE_TOO_SMALL;
  MRML_TRY(mrml_moe_ffn_prologue(hidden, attn, post_attn_norm, ffn_norm, pre_ffw_norm_2, router_scale, b.attn_res,
                                 dense ? b.shared : nullptr, b.moe_in, b.router_in, H, T, stream));
  if (dense)
    MRML_TRY(mrml_moe_dense_ffn(dense_wtype, dense_gate_up, dense_down, b.shared, b.mlp_out, H, I_dense, T, workspace,
                                b.inner, stream));
  MRML_TRY(mrml_moe_forward(wtype, router_w, b.router_in, b.moe_in, gate_up, down, down_scale, b.logits, b.ids,
                            b.probs, b.moe_out, H, I, E, K, T, workspace, b.inner, stream));
  return mrml_moe_ffn_epilogue(b.attn_res, dense ? b.mlp_out : nullptr, b.moe_out, post_ffw_norm_1, post_ffw_norm_2,
                               post_ffw_norm, hidden, layer_scale, H, T, stream);
}

int mrml_moe_rms_norm(const float* x, const float* weight, float* out, int dim, int batch, float eps,
                      mrml_stream_t stream) {
  if (dim <= 0 || batch < 0) return MRML_ERR_INVALID_ARGUMENT;
  if (batch == 0) return MRML_OK;
  if (!x || !out) return MRML_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)x & 15) != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (mrml::rms_norm_rows_per_cta(dim) == 0) return MRML_ERR_UNSUPPORTED;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_rms_norm(x, weight, out, dim, batch, eps, s));
  return MRML_OK;
}

int mrml_moe_geglu(const float* gate, const float* up, float* out, size_t n, mrml_stream_t stream) {
  if (n == 0) return MRML_OK;
  if (!gate || !up || !out || n > ((size_t)1 << 40)) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  const cudaStream_t s = (cudaStream_t)stream;
  MRML_LAUNCH(mrml::launch_geglu(gate, up, out, (long long)n, s));
  return MRML_OK;
}

int mrml_moe_quantize_q8_0(const float* src, uint8_t* dst, size_t n, mrml_stream_t stream) {
  if (n % 32 != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (n == 0) return MRML_OK;
  if (!src || !dst) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  return cuda_status(mrml::launch_quantize_gguf(kQ8_0, src, dst, (long long)(n / 32), (cudaStream_t)stream));
}

int mrml_moe_quantize_q4_0(const float* src, uint8_t* dst, size_t n, mrml_stream_t stream) {
  if (n % 32 != 0) return MRML_ERR_INVALID_ARGUMENT;
  if (n == 0) return MRML_OK;
  if (!src || !dst) return MRML_ERR_INVALID_ARGUMENT;
  MRML_TRY(check_device());
  return cuda_status(mrml::launch_quantize_gguf(kQ4_0, src, dst, (long long)(n / 32), (cudaStream_t)stream));
}

int mrml_moe_set_option(int option, int value) {
  static std::atomic<int> gv_per_sm{0}, gv_ring{0}, gv_per_sm_down{0};
  switch (option) {
    case MRML_OPTION_EXPERT_PATH:
      if (value < 0 || value > 4) return MRML_ERR_INVALID_ARGUMENT;
      g_path.store(value, std::memory_order_relaxed);
      return MRML_OK;
    case MRML_OPTION_DECODE_CTAS_PER_SM:
      if (value < 0 || value > 8) return MRML_ERR_INVALID_ARGUMENT;
      gv_per_sm.store(value);
      mrml::gv_set_tuning(gv_per_sm.load(), gv_ring.load(), gv_per_sm_down.load());
      return MRML_OK;
    case MRML_OPTION_DECODE_RING:
      if (value < 0 || value > 8) return MRML_ERR_INVALID_ARGUMENT;
      gv_ring.store(value);
      mrml::gv_set_tuning(gv_per_sm.load(), gv_ring.load(), gv_per_sm_down.load());
      return MRML_OK;
    case MRML_OPTION_DECODE_CTAS_PER_SM_DOWN:
      if (value < 0 || value > 8) return MRML_ERR_INVALID_ARGUMENT;
      gv_per_sm_down.store(value);
      mrml::gv_set_tuning(gv_per_sm.load(), gv_ring.load(), gv_per_sm_down.load());
      return MRML_OK;
    case MRML_OPTION_EXCHANGE_SPIN_LIMIT:
      if (value < 0) return MRML_ERR_INVALID_ARGUMENT;
      mrml::ep_set_spin_limit((unsigned int)value);
      return MRML_OK;
    case MRML_OPTION_L2_PREFETCH_MIB:
      if (value < 0 || value > 4096) return MRML_ERR_INVALID_ARGUMENT;
      g_prefetch_bytes.store((long long)value << 20, std::memory_order_relaxed);
      return MRML_OK;
    case MRML_OPTION_SPECULATIVE_ROUTING:
      if (value < 0 || value > 1) return MRML_ERR_INVALID_ARGUMENT;
      g_spec.store(value, std::memory_order_relaxed);
      return MRML_OK;
    default:
      return MRML_ERR_INVALID_ARGUMENT;
  }
}

int mrml_moe_profile_events(void** events, int n_events) {
  if (n_events < 0 || (n_events > 0 && !events)) return MRML_ERR_INVALID_ARGUMENT;
  t_events = n_events > 0 ? reinterpret_cast<cudaEvent_t*>(events) : nullptr;
  t_n_events = n_events;
  t_next_event = 0;
  return MRML_OK;
}

int mrml_moe_workspace_init(void* workspace, size_t workspace_bytes, mrml_stream_t stream) {
  if (!workspace || workspace_bytes < 256 || ((uintptr_t)workspace & 255u) != 0) return MRML_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaMemsetAsync(workspace, 0, 256, (cudaStream_t)stream));
}

int mrml_moe_device_status(void* workspace, mrml_stream_t stream, int* recomputed_tokens) {
  if (!workspace) return MRML_ERR_INVALID_ARGUMENT;
  int host[2] = {0, 0};
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return MRML_ERR_CUDA;
  if (cudaMemcpy(host, workspace, sizeof(host), cudaMemcpyDeviceToHost) != cudaSuccess) return MRML_ERR_CUDA;
  if (cudaMemset(workspace, 0, sizeof(host)) != cudaSuccess) return MRML_ERR_CUDA;
  if (recomputed_tokens) *recomputed_tokens = host[1];
  switch (host[0]) {
    case mrml::kDevOk: return MRML_OK;
    case mrml::kDevTimeout: return MRML_ERR_DEVICE_TIMEOUT;
    case mrml::kDevBadExpert: return MRML_ERR_BAD_EXPERT_ID;
    default: return MRML_ERR_CUDA;
  }
}

}  // extern "C"
