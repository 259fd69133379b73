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
// call); the limit and the footprint are kept as this entry point's
// published contract.  Every GPU that loads this library holds one copy of
// the array until the process exits.  All calls on a device share it, so
// calls whose kernels may overlap on the GPU (different streams without
// ordering) race on the status words; calls ordered on one stream are safe.
#include <mutex>

#include "../../include/mrml_moe.h"
#include "common.cuh"
#include "kernels.h"

constexpr size_t kNoAllocMaxBounds = 65536;
constexpr size_t kStatusFloats = 64;  // 256 bytes: [0] device status, [1] exact-fallback counter

static __device__ __align__(256) float g_router_scratch[kStatusFloats + kNoAllocMaxBounds];

namespace {

// Device address of g_router_scratch, looked up once per device (the host
// symbol is not a device address and must never be passed to a kernel).
constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MRML_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MRML_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return MRML_ERR_CUDA;
    if (major != 10) return MRML_ERR_DEVICE;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_router_scratch) != cudaSuccess || !p) return MRML_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return MRML_OK;
}

}  // namespace

extern "C" int mrml_moe_router_noalloc(const float* W, const float* x, float* logits, int32_t* ids, float* probs,
                                       int H, int E, int K, int T, mrml_stream_t stream) {
  if (H <= 0 || E <= 0 || K <= 0 || T < 0 || K > E) return MRML_ERR_INVALID_ARGUMENT;
  if (E > 256 || K > 64) return MRML_ERR_UNSUPPORTED;
  if ((size_t)T * (size_t)E > kNoAllocMaxBounds) return MRML_ERR_UNSUPPORTED;
  if (T == 0) return MRML_OK;
  if (!W || !x || !logits || !ids || !probs) return MRML_ERR_INVALID_ARGUMENT;
  float* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != MRML_OK) return st;
  const cudaStream_t s = (cudaStream_t)stream;
  int* status = reinterpret_cast<int*>(scratch);
  // The status words keep the previous call's values: clear them.
  if (cudaMemsetAsync(status, 0, kStatusFloats * sizeof(float), s) != cudaSuccess) return MRML_ERR_CUDA;
  if (mrml::launch_router_logits(W, x, logits, H, E, T, status, s) != cudaSuccess) return MRML_ERR_CUDA;
  if (mrml::launch_router_topk(logits, ids, probs, E, K, T, s) != cudaSuccess) return MRML_ERR_CUDA;
  return MRML_OK;
}
