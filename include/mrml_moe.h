/*
 * mrml_moe.h — C ABI of libmrml_moe_b200.so, the B200 (sm_100a) mixture-of-
 * experts FFN path of the MRML Gemma-4 engine.
 *
 * The library is a drop-in for the MoE operator calls of the reference's
 * Rust operator surface (crates/mrml-tensor/src/cuda.rs):
 *
 *   CudaDevice::moe_router            cuda.rs:2808-2838  -> mrml_moe_router (T = 1)
 *   CudaDevice::moe_router_batch      cuda.rs:2882-2912  -> mrml_moe_router
 *   CudaDevice::moe_topk_q4_0         cuda.rs:2772-2806  -> mrml_moe_experts (T = 1)
 *   CudaDevice::moe_topk_batch_q4_0   cuda.rs:2840-2880  -> mrml_moe_experts
 *
 * replacing the bodies of the raw launchers launch_rust_moe_router
 * (cuda.rs:849-897) and launch_rust_moe_topk (cuda.rs:1129-1220).
 *
 * Results equal the reference's CPU MoE path (model.rs:1804-1829 router,
 * model.rs:2111-2165 experts and combine): expert ids and their order are
 * bit-identical, and the layer output agrees within rel-L2 1e-4.
 *
 * Conventions
 *  - All tensor pointers are device pointers; the caller owns them.  Nothing
 *    here allocates, frees or synchronises: every call only enqueues work on
 *    `stream` and is safe to capture into a CUDA graph.
 *  - Every entry point returns MRML_OK (0) or a negative mrml_status; it
 *    never aborts the process.  A device-side failure (a bounded wait that
 *    gave up, an expert id out of range) is recorded in the workspace and
 *    read back with mrml_moe_device_status.
 *  - Shapes: H hidden size, I expert FFN size, E experts, K experts per
 *    token, T tokens.  Expert weights use the GGUF layout the reference
 *    uploads unchanged (model.rs:726-741): gate_up is [E][2I][H/32] blocks
 *    (rows [0,I) gate, [I,2I) up) and down is [E][H][I/32] blocks.
 *    H and I must be multiples of 32; weight pointers 16-byte aligned.
 *  - Limits: 1 <= K <= 64, K <= E <= 256.
 *  - Threads: calls may come from any host thread (the reference submits
 *    from one).  The options of mrml_moe_set_option are process-wide; the
 *    profiling hook is per thread; the per-device caches are thread-safe.
 *    Calls that share a workspace must be ordered on one stream.
 */
#ifndef MRML_MOE_H
#define MRML_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *mrml_stream_t; /* a cudaStream_t; NULL = legacy default stream */

typedef enum {
  MRML_OK = 0,
  MRML_ERR_INVALID_ARGUMENT = -1,  /* null pointer, bad shape, misaligned weights */
  MRML_ERR_UNSUPPORTED = -2,       /* weight type or size outside the limits above */
  MRML_ERR_WORKSPACE_TOO_SMALL = -3,
  MRML_ERR_CUDA = -4,              /* a CUDA runtime call failed; see cudaGetLastError */
  MRML_ERR_DEVICE = -5,            /* the device is not an sm_100 GPU */
  MRML_ERR_DEVICE_TIMEOUT = -6,    /* reported by mrml_moe_device_status */
  MRML_ERR_BAD_EXPERT_ID = -7,     /* reported by mrml_moe_device_status */
  MRML_ERR_NOT_FOUND = -8,         /* a GGUF tensor or metadata key that the file does not have */
} mrml_status;

/* GGML type ids (crates/mrml-tensor/src/types.rs:7-27).  MRML_PACKED or'ed
 * into a weight type marks expert weights repacked by
 * mrml_moe_prepare_weights (no counterpart in the reference). */
enum { MRML_Q4_0 = 2, MRML_Q8_0 = 8, MRML_PACKED = 0x100 };
enum { MRML_Q4_0_PACKED = MRML_Q4_0 | MRML_PACKED, MRML_Q8_0_PACKED = MRML_Q8_0 | MRML_PACKED };

/* Library version (major*10000 + minor*100 + patch). */
int mrml_moe_version(void);

/* Text for a status code (static storage). */
const char *mrml_moe_status_string(int status);

/* Bytes of device workspace that mrml_moe_router / mrml_moe_experts /
 * mrml_moe_forward need for these shapes (a multiple of 256).  The
 * workspace must be 256-byte aligned and may be reused by calls that are
 * ordered on one stream; concurrent calls need separate workspaces. */
size_t mrml_moe_workspace_bytes(int H, int I, int E, int K, int T);

/* Clears the status words at the start of a workspace (an async memset on
 * `stream`).  Call once after allocating a workspace, before its first use. */
int mrml_moe_workspace_init(void *workspace, size_t workspace_bytes, mrml_stream_t stream);

/* Router: logits[T][E] = x[T][H] . W[E][H]^T, then per token the K best
 * experts (logit descending, ties to the lower id) and their renormalised
 * softmax weights ids[T][K], probs[T][K].
 * Replaces launch_rust_moe_router (cuda.rs:849-897), which always used K=8;
 * semantics of model.rs:1804-1829.  Logits, ids and probs equal the
 * reference CPU path's bit for bit (sequential f32 dot products, glibc's
 * expf).  The workspace is only checked for size and may be shared with
 * mrml_moe_experts. */
int mrml_moe_router(const float *W, const float *x, float *logits, int32_t *ids, float *probs, int H, int E, int K,
                    int T, void *workspace, size_t workspace_bytes, mrml_stream_t stream);

/* Intervals lo[T][E] <= logits <= hi[T][E] that contain mrml_moe_router's
 * logits (the reference's sequential f32 dot products, model.rs:1804-1814),
 * computed in parallel: exact f64 products and sums plus a rigorous bound on
 * the sequential chain's rounding, rounded outward to f32.  The interval is
 * about H * 2^-24 times the mean |prefix sum| wide.  mrml_moe_forward uses it
 * to select candidate experts before the exact logits are ready (speculative
 * routing).  No counterpart in the reference.  H a multiple of 128, W and x
 * 16-byte aligned (else MRML_ERR_UNSUPPORTED). */
int mrml_moe_router_logit_bounds(const float *W, const float *x, float *lo, float *hi, int H, int E, int T,
                                 mrml_stream_t stream);

/* mrml_moe_router for callers that cannot allocate device memory.  No
 * counterpart in the reference (its router always had a device buffer set
 * up by the caller).  Some callers can only use buffers they were given:
 * a sandboxed or mediated GPU client that may launch work but not create
 * allocations, code that must not allocate on its latency path, or code
 * recording into a CUDA graph, where cudaMalloc cannot be captured.  This
 * entry point keeps the router's scratch in a fixed device array inside the
 * library, so it allocates nothing and needs no workspace argument; results
 * equal mrml_moe_router's.  Limit: T * E <= 65536, otherwise
 * MRML_ERR_UNSUPPORTED.  The array (about 256 KiB) is held on every GPU that
 * loads the library until the process exits.  The first call on a device
 * looks up the array's device address; make that first call before any
 * stream capture (calls on a stream that is
 * not capturing look the address up again, so a cudaDeviceReset between
 * calls is safe).  All calls on a device share the array (each call clears
 * its status words first), so calls whose kernels can overlap on the GPU,
 * such as calls on unordered streams, race; calls ordered on one stream are
 * fine.  A device-side failure (a bounded wait that gave up) is read with
 * mrml_moe_router_noalloc_status, not mrml_moe_device_status. */
int mrml_moe_router_noalloc(const float *W, const float *x, float *logits, int32_t *ids, float *probs, int H, int E,
                            int K, int T, mrml_stream_t stream);

/* Synchronises `stream`, then reads and clears the device status word of
 * mrml_moe_router_noalloc's array on the current device: MRML_OK or
 * MRML_ERR_DEVICE_TIMEOUT (the router's staging wait gave up; the logits of
 * the affected tokens were not written).  The word is shared by every
 * noalloc call on the device and holds the first failure since it was last
 * cleared (each mrml_moe_router_noalloc call clears it too).  No counterpart
 * in the reference.  Not capturable: returns MRML_ERR_INVALID_ARGUMENT if
 * `stream` is being captured. */
int mrml_moe_router_noalloc_status(mrml_stream_t stream);

/* Top-K and softmax from caller-supplied logits[T][E] (model.rs:1816-1829).
 * Needs no workspace. */
int mrml_moe_route_from_logits(const float *logits, int32_t *ids, float *probs, int E, int K, int T,
                               mrml_stream_t stream);

/* Experts and combine: out[T][H] = sum_k probs[t,k] * down_e(geglu(gate_e x,
 * up_e x)) * down_scale[e], with x quantised to Q8_0 and act re-quantised to
 * Q8_0 exactly as the reference CPU path does (model.rs:2111-2165); slots
 * with probs <= 1e-4 are skipped.  down_scale may be NULL (all 1.0).
 * out is overwritten (the reference's GPU path memsets and accumulates).
 * Replaces launch_rust_moe_topk (cuda.rs:1129-1220); wtype Q4_0 is the
 * reference's format, Q8_0 is an extension with the same structure. */
int mrml_moe_experts(int wtype, const uint8_t *gate_up, const uint8_t *down, const int32_t *ids, const float *probs,
                     const float *down_scale, const float *x, float *out, int H, int I, int E, int K, int T,
                     void *workspace, size_t workspace_bytes, mrml_stream_t stream);

/* One expert-parallel shard of mrml_moe_experts.  No counterpart in the
 * reference, which keeps all experts on one device.  gate_up and down hold
 * only experts [e_first, e_first + e_count) of the layer's E (same per-expert
 * layout as above, expert e_first first); ids are global in [0, E).  Pairs
 * routed to experts outside the shard are skipped like pairs with
 * alpha <= 1e-4, and out[t] is the slot-ordered sum over this shard's pairs,
 * (alpha * down) * down_scale[id] (down_scale indexed by the global id), or 0
 * for a token with none.  Summing the shards' outputs gives the layer output
 * within rounding of the single-device result (the sum order differs).
 * Workspace: mrml_moe_workspace_bytes(H, I, e_count, K, T).  Used by the
 * expert-parallel layer across GPUs, where T covers every rank's tokens. */
int mrml_moe_experts_shard(int wtype, const uint8_t *gate_up, const uint8_t *down, const int32_t *ids,
                           const float *probs, const float *down_scale, const float *x, float *out, int H, int I,
                           int E, int e_first, int e_count, int K, int T, void *workspace, size_t workspace_bytes,
                           mrml_stream_t stream);

/* Expert parallelism across the GPUs of one node, over NVLink peer memory
 * (no counterpart in the reference, which runs the layer on one device; its
 * MoE call, cuda.rs:2840-2880, becomes the per-rank expert step here).
 * Rank r of N (one process per GPU) holds experts [r*E/N, (r+1)*E/N) and T
 * home tokens.  Set-up: every rank allocates one slab of
 * mrml_moe_ep_slab_bytes(N, T, H, K) bytes with mrml_moe_ep_slab_alloc
 * (zeroed), shares its IPC handle (mrml_moe_ipc_get_handle, 64 bytes), opens
 * the others' (mrml_moe_ipc_open_handle) and keeps a device array `slabs` of
 * the N slab pointers in rank order (its own at its own index).  Per layer
 * step, after routing its home tokens (ids, probs [T][K]), every rank calls
 * on one stream, in this order:
 *   mrml_moe_ep_dispatch: quantises each home row x[t] to Q8_0 once (the
 *     layer's activation quantiser) and stores it into the slabs of the ranks
 *     that own one of t's experts (pairs with probs > 1e-4), with the ids and
 *     weights of every home token into every rank;
 *   mrml_moe_ep_experts: waits for all N ranks' dispatch, runs this rank's
 *     experts (gate_up / down hold experts [r*E/N, (r+1)*E/N) only, in the
 *     layout of mrml_moe_experts; down_scale, if given, is indexed by global
 *     id) on the received rows, and stores into each token's home rank the
 *     slot-ordered partial sum over this rank's pairs of it;
 *   mrml_moe_ep_combine: waits for all N ranks' partials, then out[T][H] =
 *     for each home token, its partials summed in rank order (0 for a token
 *     with no pair).
 * The output equals the single-device layer within rounding: each rank's
 * partial is the single-device slot-ordered sum restricted to its pairs, and
 * the partials are then added in rank order (bit-identical when one rank owns
 * all of a token's experts).  Nothing synchronises with the host, so a whole
 * step can be captured in a CUDA graph.  Waits are bounded (see
 * MRML_OPTION_EXCHANGE_SPIN_LIMIT); a wait that gives up writes
 * MRML_ERR_DEVICE_TIMEOUT's device code into the workspace's status word
 * (read with mrml_moe_device_status) and leaves the data it would have
 * produced untouched.  All ranks must make the same calls with the same
 * shapes; H a multiple of 32, x 16-byte aligned, E a multiple of N, N <= 16; the experts need
 * the decode kernel's shapes (H a multiple of 256, I of 64).  The workspace
 * (mrml_moe_ep_workspace_bytes, 256-byte aligned, zeroed once with
 * mrml_moe_workspace_init) serves mrml_moe_ep_experts and
 * mrml_moe_ep_combine. */
size_t mrml_moe_ep_slab_bytes(int N, int T, int H, int K);
size_t mrml_moe_ep_workspace_bytes(int N, int T, int H, int I, int E, int K);
int mrml_moe_ep_slab_alloc(size_t bytes, void **slab);
int mrml_moe_ep_slab_free(void *slab);
int mrml_moe_ipc_get_handle(const void *slab, void *handle);
int mrml_moe_ipc_open_handle(const void *handle, void **slab);
int mrml_moe_ipc_close_handle(void *slab);
int mrml_moe_ep_dispatch(void *const *slabs, int rank, int N, int T, int H, int E, int K, const float *x,
                         const int32_t *ids, const float *probs, mrml_stream_t stream);
int mrml_moe_ep_experts(int wtype, const uint8_t *gate_up, const uint8_t *down, const float *down_scale,
                        void *const *slabs, int rank, int N, int T, int H, int I, int E, int K, void *workspace,
                        size_t workspace_bytes, mrml_stream_t stream);
int mrml_moe_ep_combine(void *const *slabs, int rank, int N, int T, int H, int E, int K, const int32_t *ids,
                        const float *probs, float *out, void *workspace, mrml_stream_t stream);

/* The whole layer: mrml_moe_router on (router_w, router_x) followed by
 * mrml_moe_experts on x.  router_x and x may be the same pointer.  Up to 32
 * tokens (E <= 256, K <= 64) the experts' dispatch kernel selects the
 * experts itself from the logits (the same selection code, one launch
 * fewer); logits, ids and probs are written either way. */
int mrml_moe_forward(int wtype, const float *router_w, const float *router_x, const float *x, const uint8_t *gate_up,
                     const uint8_t *down, const float *down_scale, float *logits, int32_t *ids, float *probs,
                     float *out, int H, int I, int E, int K, int T, void *workspace, size_t workspace_bytes,
                     mrml_stream_t stream);

/* Bytes of one layer's expert weights: which = 0 gate_up ([E][2I][H/32]
 * blocks), 1 down ([E][H][I/32] blocks); the same for the GGUF layout and
 * the packed one.  0 for an invalid shape. */
size_t mrml_moe_weights_bytes(int wtype, int H, int I, int E, int which);

/* Load-time repack of one layer's GGUF expert weights (the slabs the
 * reference uploads unchanged, model.rs:726-741, read from the GGUF file at
 * model.rs:630-755) into the layout the decode expert kernel reads fastest:
 * the same bytes (same size), reordered so that every lane of the warp-level
 * MMA reads its weight fragment and both rows' f16 scales with aligned vector
 * loads.  Pass the packed buffers to mrml_moe_experts / _forward / _shard
 * with wtype | MRML_PACKED; results are bit-identical to the GGUF layout's.
 * No counterpart in the reference (its GPU path reads the raw blocks).
 * wtype MRML_Q4_0 or MRML_Q8_0; outputs mrml_moe_weights_bytes each, 16-byte
 * aligned, not overlapping the inputs.  Needs H a multiple of 256 and I of
 * 64 (MRML_ERR_UNSUPPORTED otherwise).  Enqueued on `stream`; capturable. */
int mrml_moe_prepare_weights(int wtype, const uint8_t *gate_up, const uint8_t *down, uint8_t *gate_up_packed,
                             uint8_t *down_packed, int H, int I, int E, mrml_stream_t stream);

/* GGUF v2/v3 tensor table (host code), for loading the MoE layers' expert
 * slabs as the reference's loader does: gguf.rs:80-181 parses the header,
 * metadata and tensor infos (the data section starts at the next multiple of
 * general.alignment, default 32), and model.rs:638-647 takes a tensor at
 * data_offset + offset, e.g. "blk.{l}.ffn_gate_up_exps.weight" and
 * "blk.{l}.ffn_down_exps.weight", whose bytes model.rs:726-741 uploads
 * unchanged.  mrml_moe_gguf_open reads the header of the file at `path`
 * (MRML_ERR_UNSUPPORTED for another version or a tensor type the reference
 * does not read); mrml_moe_gguf_tensor gives a tensor's GGML type, dimensions
 * (up to 4, innermost first), absolute file offset and size in bytes
 * (elements / block elements * block bytes); mrml_moe_gguf_meta_u32 an
 * integer metadata value; mrml_moe_gguf_read copies a tensor's bytes into a
 * host buffer.  Missing names return MRML_ERR_NOT_FOUND.  The handle is
 * read-only after opening and may be shared between threads. */
int mrml_moe_gguf_open(const char *path, void **file);
int mrml_moe_gguf_close(void *file);
int mrml_moe_gguf_version(const void *file);
int mrml_moe_gguf_tensor_count(const void *file);
const char *mrml_moe_gguf_tensor_name(const void *file, int i);
int mrml_moe_gguf_tensor(const void *file, const char *name, int *ggml_type, int *n_dims, int64_t *dims,
                         uint64_t *file_offset, uint64_t *nbytes);
int mrml_moe_gguf_meta_u32(const void *file, const char *key, uint32_t *value);
int mrml_moe_gguf_read(const void *file, const char *name, void *dst, size_t dst_bytes);

/* The weighted combine alone (model.rs:2163-2165): out[t][i] = sum over
 * k ascending of (probs[t,k] * ydown[pos[t,k]][i]) * down_scale[ids[t,k]],
 * starting from 0; pairs with pos < 0 are skipped.  ydown holds unscaled
 * down-projection rows, one per (token, slot).  Used by the expert-parallel
 * path, where those rows come back from the ranks that own the experts. */
int mrml_moe_combine(const float *ydown, const int32_t *pos, const int32_t *ids, const float *probs,
                     const float *down_scale, float *out, int H, int K, int T, mrml_stream_t stream);

/* The FFN prologue of a Gemma-4 MoE layer, fused: replaces
 * launch_rust_prepare_ffn (cuda.rs:899-949, kernel rust_cuda_prepare_ffn_f32
 * in cuda_ptx/kernels.rs:987-1033) with the same arguments, and computes
 * what the reference's CPU path does (model.rs:1719-1784) bit for bit.
 * Per row of `dim` floats (batch rows), eps 1e-6:
 *   attn_res = hidden + rms_norm(attn, post_attn_norm)
 *   shared   = rms_norm(attn_res, ffn_norm)          the shared dense MLP's input
 *   moe      = rms_norm(attn_res, pre_ffw_norm_2)    the experts' input
 *   router   = rms_norm(attn_res) * (1 / sqrt(dim)) * router_scale
 * rms_norm as ops.rs:24-49 (sequential sum of squares, (x * s) * w).
 * Extensions: attn NULL takes hidden as the residual; any output may be NULL
 * (not written); a NULL weight means 1.  dim <= 51200. */
int mrml_moe_ffn_prologue(const float *hidden, const float *attn, const float *post_attn_norm,
                          const float *ffn_norm, const float *pre_ffw_norm_2, const float *router_scale,
                          float *attn_res, float *shared, float *moe, float *router, int dim, int batch,
                          mrml_stream_t stream);

/* The FFN epilogue, fused: replaces launch_rust_finish_ffn (cuda.rs:951-987,
 * kernel rust_cuda_finish_ffn_f32 in cuda_ptx/kernels.rs:1036-1083) with the
 * same arguments; the CPU path's arithmetic (model.rs:2176-2196):
 *   output = (attn_res + rms_norm(rms_norm(dense, post_ffw_norm_1)
 *                                 + rms_norm(moe, post_ffw_norm_2), post_ffw_norm))
 *            * layer_scale
 * Unlike the reference's kernel it leaves dense and moe unchanged.  dense
 * may be NULL (a layer without the shared MLP: zeros); a NULL weight means
 * 1; output may alias attn_res.  dim <= 25600. */
int mrml_moe_ffn_epilogue(const float *attn_res, const float *dense, const float *moe,
                          const float *post_ffw_norm_1, const float *post_ffw_norm_2, const float *post_ffw_norm,
                          float *output, float layer_scale, int dim, int batch, mrml_stream_t stream);

/* The layer's shared dense GeGLU MLP (model.rs:2093-2109 on the CPU;
 * gemv_q4_0_geglu + gemv_q4_0 on the reference's GPU, model.rs:1889-1890):
 * out[T][H] = down(geglu(gate x, up x)) with x and act quantised to Q8_0 as
 * the reference does, bit-identical to it.  It is the expert arithmetic of
 * mrml_moe_experts for one expert with weight 1, so gate_up holds the
 * ffn_gate rows then the ffn_up rows ([2I][H/32] blocks) and down [H][I/32]
 * blocks; packed weights (mrml_moe_prepare_weights with E = 1) are taken
 * too.  Run it on a second stream to overlap it with the MoE experts, as the
 * reference's captured layer does.  Workspace:
 * mrml_moe_dense_ffn_workspace_bytes. */
size_t mrml_moe_dense_ffn_workspace_bytes(int H, int I, int T);
int mrml_moe_dense_ffn(int wtype, const uint8_t *gate_up, const uint8_t *down, const float *x, float *out, int H,
                       int I, int T, void *workspace, size_t workspace_bytes, mrml_stream_t stream);

/* One whole FFN block of a Gemma-4 MoE layer on the device-resident hidden
 * state, in one capturable call (the body of the reference's captured
 * per-layer FFN graph, capture_layer_ffn_graph model.rs:295-381 /
 * enqueue_ffn_compute_for_capture cuda.rs:1885-1955, with the prepare and
 * finish steps around it, model.rs:1719-2196):
 *   mrml_moe_ffn_prologue(hidden, attn, ...) -> residual, MLP / MoE / router
 *   inputs; mrml_moe_dense_ffn (if I_dense > 0); mrml_moe_forward;
 *   mrml_moe_ffn_epilogue -> hidden (overwritten in place).
 * Everything between lives in the workspace
 * (mrml_moe_ffn_block_workspace_bytes, 256-byte aligned, cleared once with
 * mrml_moe_workspace_init; mrml_moe_device_status reads its status word).
 * dense_wtype is the shared MLP's weight type (its slabs as for
 * mrml_moe_dense_ffn).  Bit-identical to the reference's CPU block.  Capture
 * it once per layer and replay the graph per decode step. */
size_t mrml_moe_ffn_block_workspace_bytes(int H, int I, int I_dense, int E, int K, int T);
int mrml_moe_ffn_block(int wtype, int dense_wtype, float *hidden, const float *attn, const float *post_attn_norm,
                       const float *ffn_norm, const float *pre_ffw_norm_2, const float *router_scale,
                       const float *post_ffw_norm_1, const float *post_ffw_norm_2, const float *post_ffw_norm,
                       float layer_scale, const float *router_w, const uint8_t *gate_up, const uint8_t *down,
                       const float *down_scale, const uint8_t *dense_gate_up, const uint8_t *dense_down, int H, int I,
                       int I_dense, int E, int K, int T, void *workspace, size_t workspace_bytes,
                       mrml_stream_t stream);

/* RMS normalisation of `batch` rows of `dim` floats: out = x / sqrt(mean(x^2)
 * + eps) * weight (weight may be NULL), with the reference's rounding: the
 * sum of squares in index order, then 1 / sqrt(sum / dim + eps) (ops.rs:24-49;
 * the norm applied after the MoE output, model.rs:2176-2196).  Replaces
 * CudaDevice::rms_norm_batch (cuda.rs:2139) and rms_norm (cuda.rs:2102) with
 * the same argument order.  x 16-byte aligned; dim <= 51200; out may not
 * alias x. */
int mrml_moe_rms_norm(const float *x, const float *weight, float *out, int dim, int batch, float eps,
                      mrml_stream_t stream);

/* GeGLU, elementwise: out[i] = gelu_tanh(gate[i]) * up[i] with the
 * reference's formula and rounding (ops.rs:99-114; tanh as glibc's tanhf),
 * the expert epilogue applied on its own.  Replaces CudaDevice::geglu
 * (crates/mrml-tensor/src/cuda.rs:2215), the launch of rust_cuda_geglu_f32. */
int mrml_moe_geglu(const float *gate, const float *up, float *out, size_t n, mrml_stream_t stream);

/* GGUF block quantisers on the device, byte-identical to the reference's
 * host quantisers: Q8_0 quant.rs:193-228, Q4_0 quant.rs:372-389.
 * n is a multiple of 32; dst holds n/32*34 (Q8_0) or n/32*18 (Q4_0) bytes. */
int mrml_moe_quantize_q8_0(const float *src, uint8_t *dst, size_t n, mrml_stream_t stream);
int mrml_moe_quantize_q4_0(const float *src, uint8_t *dst, size_t n, mrml_stream_t stream);

/* Process-wide options.  MRML_OPTION_EXPERT_PATH selects how the expert
 * products run: 0 automatic (the pipelined kernel with warp-level MMA from 2
 * tokens per expert, else the same kernel with dp4a dots; when that
 * kernel's shape limits are not met (H a multiple of 256, I of 64), the
 * general kernels, or tcgen05 above 16 tokens per expert),
 * 1 pipelined decode kernel with dp4a, 2 tensor cores, 3 the general
 * CUDA-core kernels (any H, I multiple of 32; used automatically when H is
 * not a multiple of 256), 4 pipelined decode kernel with warp-level MMA.
 * All paths give bit-identical results; the option exists for tests and
 * benchmarks. */
enum { MRML_OPTION_EXPERT_PATH = 1 };
/* Tuning of the decode (CUDA-core) expert kernel: CTAs per SM (1..8) and
 * the depth of its weight ring (1..8); 0 restores the automatic choice. */
enum { MRML_OPTION_DECODE_CTAS_PER_SM = 2, MRML_OPTION_DECODE_RING = 3 };
/* CTAs per SM of the down product alone (1..8; 0: as the option above). */
enum { MRML_OPTION_DECODE_CTAS_PER_SM_DOWN = 7 };
/* Poll limit of the expert-parallel exchange's bounded waits (about 2^24 by
 * default, over a second; 0 restores the default).  Lets a test make a wait
 * give up quickly. */
enum { MRML_OPTION_EXCHANGE_SPIN_LIMIT = 4 };
/* Speculative routing in mrml_moe_forward (and the FFN block) for batches of
 * at most 32 tokens: 0 off (default), 1 on.  The dispatch then selects, from
 * intervals that bound the router logits' rounding
 * (mrml_moe_router_logit_bounds), the experts that can be in the top-K, and
 * the exact router runs on a library-owned stream beside the expert
 * products; results are identical either way.  Off by default: on B200 the
 * join of the two streams cost about what the shorter critical path saved. */
enum { MRML_OPTION_SPECULATIVE_ROUTING = 5 };
/* MiB of expert gate/up weights that mrml_moe_forward's router launch asks
 * the L2 to fetch ahead (0..4096; default 64) when the batch is likely to
 * hit nearly every expert (T * K >= 2 E, T <= 256): the experts the products
 * read first, fetched while routing leaves the HBM idle.  A cache hint;
 * results do not depend on it. */
enum { MRML_OPTION_L2_PREFETCH_MIB = 6 };
int mrml_moe_set_option(int option, int value);

/* Profiling hook for benchmarks.  With n_events > 0, the following calls on
 * this host thread record events[2i] (a cudaEvent_t) on their stream just
 * before their i-th kernel launch and events[2i+1] just after it, counting
 * launches across calls, until the list is used up or the hook is reset
 * with mrml_moe_profile_events(NULL, 0).  Per call: mrml_moe_router 2
 * launches (router_logits, router_topk), mrml_moe_route_from_logits 1,
 * mrml_moe_experts 5 (dispatch, quantize, gate_up, down, combine) — 6 from
 * 256 tokens on the decode kernels (quantize_rows, dispatch, gather, gate_up,
 * down, combine) — and mrml_moe_forward the router's 2 plus those, or 6 up to
 * 32 tokens (router_logits, then the dispatch kernel with the selection, then
 * the other four). */
int mrml_moe_profile_events(void **events, int n_events);

/* Synchronises `stream`, reads and clears the device status word of a
 * workspace: MRML_OK, MRML_ERR_DEVICE_TIMEOUT or MRML_ERR_BAD_EXPERT_ID.
 * recomputed_tokens is deprecated: it may be NULL, and otherwise always
 * receives 0 (the router computes every logit exactly and has no fallback
 * to count; the argument stays for binary compatibility and will be removed
 * at the next major version).  Not capturable. */
int mrml_moe_device_status(void *workspace, mrml_stream_t stream, int *recomputed_tokens);

#ifdef __cplusplus
}
#endif
#endif /* MRML_MOE_H */
