// kernels.h — host launchers of the MRML MoE kernels (internal).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace mrml {

// Shape limits shared by every entry point (the top-k keeps up to 256
// experts in a warp's registers and up to 64 candidates in shared memory).
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 64;
// Devices whose per-device host caches are kept (higher ordinals work, but
// repeat the cached lookups on every call).
constexpr int kMaxDevices = 64;

// The dynamic shared memory a kernel has been opened up to on each device.
// cudaFuncSetAttribute is host-side state, not a stream operation; calling
// it once per (kernel, device, size) keeps it off the decode path's host
// time.  Safe to call from several host threads: the fast path reads an
// atomic, and the attribute only ever grows (under a lock), so a thread
// cannot lower the limit another thread is about to launch with.
struct SmemOptIn {
  std::atomic<int> bytes[kMaxDevices];
};
inline std::mutex& smem_opt_in_lock() {
  static std::mutex m;
  return m;
}
template <typename Kern>
inline cudaError_t ensure_smem(Kern k, size_t bytes, SmemOptIn& c) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  const bool cached = dev >= 0 && dev < kMaxDevices;
  if (cached && c.bytes[dev].load(std::memory_order_acquire) >= (int)bytes) return cudaSuccess;
  std::lock_guard<std::mutex> lock(smem_opt_in_lock());
  const int target = cached ? std::max((int)bytes, c.bytes[dev].load(std::memory_order_relaxed)) : (int)bytes;
  st = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, target);
  if (st == cudaSuccess && cached) c.bytes[dev].store(target, std::memory_order_release);
  return st;
}

// Launches `kern` with programmatic dependent launch: the grid may start
// while the previous kernel on the stream finishes (its CTAs run their
// prologue, then wait in pdl_wait() for the previous grid to complete and
// its writes to be visible).  Every kernel of the library calls pdl_wait()
// before its first read of anything an earlier kernel wrote, and
// pdl_trigger() once its own CTAs are running.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// With prefetch_bytes > 0 (a multiple of 16, `prefetch` 16-byte aligned),
// the decode-size router kernel also asks the L2 for those bytes (a hint for
// the expert products that follow; ignored by the large-batch kernels).
cudaError_t launch_router_logits(const float* W, const float* x, float* logits, int H, int E, int T, int* err,
                                 cudaStream_t s, const uint8_t* prefetch = nullptr, size_t prefetch_bytes = 0);
cudaError_t launch_router_topk(const float* logits, int32_t* ids, float* probs, int E, int K, int T, cudaStream_t s);
// Intervals [lo, hi] (f32, [T][E]) that contain the reference's router
// logits, from parallel f64 sums and a rigorous bound on the sequential f32
// chain's rounding (router.cu); H a multiple of 128, 16-byte aligned rows.
bool router_bounds_supported(const float* W, const float* x, int H);
cudaError_t launch_router_bounds(const float* W, const float* x, float* lo, float* hi, int H, int E, int T, int* err,
                                 cudaStream_t s);
cudaError_t launch_quantize_rows(const float* x, int8_t* xq, float* xd, int32_t* xsum, long long n_blocks,
                                 cudaStream_t s);
cudaError_t launch_quantize_gguf(int wtype, const float* x, uint8_t* dst, long long n_blocks, cudaStream_t s);
int rms_norm_rows_per_cta(int H);
cudaError_t launch_rms_norm(const float* x, const float* w, float* out, int H, int T, float eps, cudaStream_t s);
cudaError_t launch_ffn_prologue(const float* hidden, const float* attn, const float* pan, const float* ffn_norm,
                                const float* pre_norm2, const float* gis, float* attn_res, float* x_shared,
                                float* x_moe, float* router_x, int H, int T, float eps, cudaStream_t s);
cudaError_t launch_ffn_epilogue(const float* attn_res, const float* mlp_raw, const float* moe_raw, const float* post1,
                                const float* post2, const float* post, float out_scale, float* hidden, int H, int T,
                                float eps, cudaStream_t s);
cudaError_t launch_geglu(const float* gate, const float* up, float* out, long long n, cudaStream_t s);
cudaError_t launch_dense_routing(int32_t* ids, float* probs, int T, cudaStream_t s);
// Speculative selection (small batches): the router logits' intervals
// [lo, hi] ([T][E], launch_router_bounds), the router's weights [E][H] and
// inputs [T][H] for tokens whose intervals do not settle the choice, the
// reference's K and the candidate slots C per token (K <= C <= E).
struct SpecRoute {
  const float* lo;
  const float* hi;
  const float* W;
  const float* x;
  int H, K, C;
};
cudaError_t launch_dispatch(const int32_t* ids, const float* probs, int n_pairs, int E, int e_first, int e_total,
                            int32_t* cnt, int32_t* poff,
                            int32_t* pair_at, int32_t* pos, int4* units_gu, int4* units_dn, int* n_units,
                            int NT_gu, int NT_dn, int mt_gu, int rows_gu, int mt_dn, int* err, cudaStream_t s,
                            const float* logits = nullptr, int K = 0, int32_t* ids_out = nullptr,
                            float* probs_out = nullptr, int32_t* chunk_cnt = nullptr,
                            const SpecRoute* spec = nullptr);
// Candidate slots per token of the speculative selection: K plus a few for
// experts whose logits lie within the rounding bound of the K-th.
constexpr int kSpecExtraSlots = 4;
inline int spec_slots(int E, int K) { return K + kSpecExtraSlots < E ? K + kSpecExtraSlots : E; }
// Above this many pairs (and with chunk_cnt, dispatch_chunk_ints(n_pairs, E)
// ints of scratch) the dispatch runs as three launches over chunks of 1024
// pairs instead of one CTA; same result.
constexpr int kDispatchChunkedMin = 8192;
inline size_t dispatch_chunk_ints(long long n_pairs, int E) { return (size_t)((n_pairs + 1023) / 1024) * E; }
// Whether launch_dispatch can select the experts itself (from `logits`) for
// T tokens: the top-k of up to 256 experts for up to kDispatchTopkMaxTokens
// tokens.
constexpr int kDispatchTopkMaxTokens = 32;
// Batches with T * E up to this select by rank inside the dispatch kernel.
constexpr int kDispatchRankSelectMax = 512;
bool dispatch_topk_supported(int E, int K, int T);
// The decode kernel's group-major operand from the per-token quantisation
// (xq/xd/xsum of launch_quantize_rows) and the dispatch's pair_at; poff_end
// is the device count of positions in use.
cudaError_t launch_gather_groups(int wtype, const int8_t* xq, const float* xd, const int32_t* xsum,
                                 const int32_t* pair_at, const int32_t* poff_end, int H, int K, int npad, int8_t* bq,
                                 int2* bsc, cudaStream_t s);
cudaError_t launch_quantize_scatter(int wtype, const float* x, const int32_t* pos, int T, int H, int K, int npad,
                                    bool group_major, int8_t* bq, int2* bsc, cudaStream_t s);
cudaError_t launch_gate_up(int wtype, const uint8_t* gate_up, const int32_t* cnt, const int32_t* poff,
                           const int32_t* sorted, const int8_t* xq, const float* xd, const int32_t* xsum, float* act,
                           int H, int I, int E, int K, int* err, cudaStream_t s);
cudaError_t launch_down(int wtype, const uint8_t* down, const int32_t* cnt, const int32_t* poff, const float* act,
                        float* ydown, int H, int I, int E, int* err, cudaStream_t s);
// Tensor-core grouped products (gemm_tc.cu).  mode 0 = gate/up, 1 = down.
bool tc_map_available();
bool tc_make_gate_up_map(CUtensorMap* m, const uint8_t* w, int wtype, int H, int I, int E, int box_rows);
int tc_num_sms();
// CUDA-core pipelined products for decode-size tiles (gemv.cu): units of
// kGvTokens positions and kGvRowsGateUp gate (and as many up) rows, or
// 2 * kGvRowsGateUp down rows; otherwise the same arguments as
// launch_gemm_tc.
constexpr int kGvTokens = 8;
constexpr int kGvRowsGateUp = 64;
bool gv_supported(int wtype, int H, int I);
void gv_set_tuning(int per_sm, int ring, int per_sm_down);
// ng: position groups of 8 per work unit (1, or 2 on the MMA form);
// packed: the weights are in mrml_moe_prepare_weights' layout.
// per_sm > 0 asks for that many CTAs per SM (at most the kernel's bound;
// the tuning options still take precedence); 0 chooses automatically.
cudaError_t launch_gemv(int mode, int wtype, bool packed, bool mma, int ng, const uint8_t* weights, int H, int I,
                        int E, const int8_t* bq, const int2* bsc, const int4* units, const int* n_units, int max_units,
                        int npad, int8_t* out_q, int2* out_s, float* y, int* err, cudaStream_t s, int per_sm = 0);
// Whether the packed layout (and the decode kernel on it) fits these shapes.
bool gv_packed_supported(int wtype, int H, int I);
// Repacks raw GGUF expert weights into the decode kernel's packed layout
// (prepare.cu); which = 0 gate_up [E][2I][H/32 blocks], 1 down [E][H][I/32].
cudaError_t launch_repack(int which, int wtype, const uint8_t* src, uint8_t* dst, int H, int I, int E,
                          cudaStream_t s);
// Whether the MMA form's 16-position units fit these shapes.
bool gv_two_groups_supported(int wtype, int H, int I);
bool tc_supported(int wtype, int H, int I, int NT);
cudaError_t launch_gemm_tc(int mode, int wtype, int NT, const uint8_t* weights, int H, int I, int E, const int8_t* bq,
                           const int2* bsc, const int4* units, const int* n_units, int max_units, int npad,
                           int8_t* out_q, int2* out_s, float* y, int* err, cudaStream_t s);
cudaError_t launch_combine(const float* ydown, const int32_t* pos, const int32_t* ids, const float* probs,
                           const float* down_scale, float* out, int H, int K, int T, cudaStream_t s);
// Combine after a speculative dispatch: pos and cand are [T][C] (the
// candidates' positions and expert ids); each of the reference's K slots
// (ids / probs, [T][K]) finds its expert among the token's candidates.  A
// slot whose expert is missing sets the status word's bad-expert code.
cudaError_t launch_combine_spec(const float* ydown, const int32_t* pos, const int32_t* cand, const int32_t* ids,
                                const float* probs, const float* down_scale, float* out, int H, int K, int C, int T,
                                int* err, cudaStream_t s);

// Expert-parallel exchange over peer memory (ep_p2p.cu).
constexpr int kEpMaxRanks = 16;
size_t ep_slab_bytes(int N, int T, int H, int K);
// Poll limit of the exchange's bounded waits (0 restores the default).
void ep_set_spin_limit(unsigned int limit);
cudaError_t launch_ep_dispatch(uint8_t* const* slabs, int rank, int N, int T, int H, int E, int K, const float* x,
                               const int32_t* ids, const float* probs, cudaStream_t s);
cudaError_t launch_ep_recv(uint8_t* const* slabs, int rank, int N, int T, int H, int K, int32_t* ids_all,
                           float* probs_all, const uint8_t** rows, int* err, cudaStream_t s);
cudaError_t launch_ep_gather(int wtype, const uint8_t* const* rows, const int32_t* pair_at, const int32_t* poff_end,
                             int H, int K, int npad, int8_t* bq, int2* bsc, cudaStream_t s);
cudaError_t launch_ep_combine_push(uint8_t* const* slabs, int rank, int N, int T, int H, int K, const float* ydown,
                                   const int32_t* pos, const int32_t* ids_all, const float* probs_all,
                                   const float* down_scale, cudaStream_t s);
cudaError_t launch_ep_reduce(uint8_t* const* slabs, int rank, int N, int T, int H, int E, int K, const int32_t* ids,
                             const float* probs, float* out, int* err, cudaStream_t s);
int gate_up_tok_chunk(int wtype, int H);
int down_tok_chunk(int wtype, int I);

}  // namespace mrml
