// router_static.cu — the router without a caller-supplied workspace.
//
// mrml_moe_router takes a caller-allocated workspace.  Some callers cannot
// provide one: a host that only holds buffers it was handed (a sandboxed or
// mediated GPU client that may launch work but not create allocations),
// code that must not allocate on its latency path, or a caller recording
// work into a CUDA graph, where cudaMalloc is not a capturable operation.
// For them, mrml_moe_router_noalloc keeps its scratch in a fixed, file-scope
// device array instead, so the call itself allocates nothing.
//
// The array is g_router_scratch below: 256 bytes of status words followed by
// room for kNoAllocMaxBounds floats of per-(token, expert) scratch, which
// fixes the entry point's limit T * E <= 65536.  The current router kernels
// compute every logit with the reference's sequential chain and need no
// per-pair scratch, so only the status words are touched (cleared on every
// call; read and cleared by mrml_moe_router_noalloc_status); the limit and
// the footprint are kept as this entry point's published contract.  Every
// GPU that loads this library holds one copy of the array until the process
// exits.  All calls on a device share it, so calls whose kernels may overlap
// on the GPU (different streams without ordering) race on the status words;
// calls ordered on one stream are safe.
#include <atomic>
#include <mutex>

#include "../../include/mrml_moe.h"
#include "checks.h"
#include "common.cuh"
#include "kernels.h"

constexpr size_t kNoAllocMaxBounds = 65536;
constexpr size_t kStatusFloats = 64;  // 256 bytes: word 0 is the device status, the rest stay 0

static __device__ __align__(256) float g_router_scratch[kStatusFloats + kNoAllocMaxBounds];

namespace {

// Device address of g_router_scratch, looked up per device (the host symbol
// is not a device address and must never be passed to a kernel).  The first
// lookup on a device may load the library's device code, which cannot happen
// during stream capture, so the first call on each device must come before
// any capture.  The cached address does not survive cudaDeviceReset (the
// module is reloaded, possibly elsewhere), so calls on a stream that is not
// being captured look the address up again, which is cheap once loaded.
std::atomic<float*> g_scratch_ptr[mrml::kMaxDevices];
std::mutex g_scratch_mu;

int scratch_for_current_device(bool refresh, float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MRML_ERR_CUDA;
  if (dev < 0 || dev >= mrml::kMaxDevices) return MRML_ERR_DEVICE;
  float* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p && !refresh) {
    *out = p;
    return MRML_OK;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return MRML_ERR_CUDA;
  if (major != 10) return MRML_ERR_DEVICE;
  void* q = nullptr;
  if (cudaGetSymbolAddress(&q, g_router_scratch) != cudaSuccess || !q) return MRML_ERR_CUDA;
  g_scratch_ptr[dev].store(static_cast<float*>(q), std::memory_order_release);
  *out = static_cast<float*>(q);
  return MRML_OK;
}

bool capturing(cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone;
}

}  // namespace

extern "C" int mrml_moe_router_noalloc(const float* W, const float* x, float* logits, int32_t* ids, float* probs,
                                       int H, int E, int K, int T, mrml_stream_t stream) {
  const int chk = mrml::check_router_args(W, x, logits, ids, probs, H, E, K, T);
  if (chk != MRML_OK) return chk;
  if ((size_t)T * (size_t)E > kNoAllocMaxBounds) return MRML_ERR_UNSUPPORTED;
  if (T == 0) return MRML_OK;
  const cudaStream_t s = (cudaStream_t)stream;
  float* scratch = nullptr;
  const int st = scratch_for_current_device(!capturing(s), &scratch);
  if (st != MRML_OK) return st;
  int* status = reinterpret_cast<int*>(scratch);
  // The status words keep the previous call's values: clear them.
  if (cudaMemsetAsync(status, 0, kStatusFloats * sizeof(float), s) != cudaSuccess) return MRML_ERR_CUDA;
  if (mrml::launch_router_logits(W, x, logits, H, E, T, status, s) != cudaSuccess) return MRML_ERR_CUDA;
  if (mrml::launch_router_topk(logits, ids, probs, E, K, T, s) != cudaSuccess) return MRML_ERR_CUDA;
  return MRML_OK;
}

extern "C" int mrml_moe_router_noalloc_status(mrml_stream_t stream) {
  const cudaStream_t s = (cudaStream_t)stream;
  if (capturing(s)) return MRML_ERR_INVALID_ARGUMENT;
  float* scratch = nullptr;
  const int st = scratch_for_current_device(true, &scratch);
  if (st != MRML_OK) return st;
  int word = 0;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MRML_ERR_CUDA;
  if (cudaMemcpy(&word, scratch, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess) return MRML_ERR_CUDA;
  if (cudaMemsetAsync(scratch, 0, sizeof(word), s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
    return MRML_ERR_CUDA;
  switch (word) {
    case mrml::kDevOk: return MRML_OK;
    case mrml::kDevTimeout: return MRML_ERR_DEVICE_TIMEOUT;
    case mrml::kDevBadExpert: return MRML_ERR_BAD_EXPERT_ID;
    default: return MRML_ERR_CUDA;
  }
}
