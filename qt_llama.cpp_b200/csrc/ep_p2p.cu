// ep_p2p.cu — the expert-parallel exchange over NVLink peer memory.
//
// The expert-parallel layer (rank r of N holds experts [r*E/N, (r+1)*E/N)
// and T home tokens) needs two exchanges per step: every rank must see all
// N*T tokens (rows, expert ids, weights) before its experts run, and every
// token's N partial outputs must come back to its home rank and be summed.
// Here both are done by this library's kernels writing straight into the
// other GPUs' memory (CUDA IPC mappings of each rank's "slab"), without a
// collective library:
//
//   dispatch:  push   — rank r stores its home rows, ids and weights into
//                       slot r of every rank's receive area, then raises a
//                       counter in every rank's slab (system-scope atomics);
//              gather — a rank waits until all N counters show this step,
//                       then copies the N slots into the contiguous
//                       [N*T, ...] buffers its expert kernels read;
//   combine:   push   — rank r stores the partial output rows of rank q's
//                       tokens into slot r of q's partial area, then raises
//                       q's combine counter;
//              reduce — the home rank waits for all N partials and sums
//                       them in rank order (out = ((p0 + p1) + p2) + ...).
//
// Slab layout (identical on every rank, offsets from slab_layout): control
// counters written by peers, rank-local counters, and double-buffered
// receive areas indexed by the parity of the rank's step count.  Counters
// only grow (each source adds 1 per step), so no reset is needed and a step
// waits for "count >= step + 1".  The step count lives in device memory and
// every kernel reads it, so a captured step replays correctly.  Double
// buffering makes slot reuse safe: a rank writes parity p of a peer's areas
// in step s + 2 only after it has waited, in step s + 1, for that peer's
// step s + 1 combine push, which the peer issues after it finished reading
// parity p in step s.
//
// Every wait is bounded (kSpinLimit polls with back-off); a wait that gives
// up records MRML_ERR_DEVICE_TIMEOUT in the caller's status word and the
// kernel leaves without touching the data, so a rank that stops never
// hangs the others' GPUs.
#include <string.h>

#include "../../include/mrml_moe.h"
#include "common.cuh"

namespace mrml {
namespace ep {

constexpr int kMaxRanks = 16;

struct Control {
  unsigned int disp[kMaxRanks];  // dispatch pushes received from each rank
  unsigned int comb[kMaxRanks];  // combine pushes received from each rank
  unsigned int step;             // steps completed by this rank (rank-local)
  unsigned int done_push;        // CTAs of the running push kernel that finished (rank-local)
  unsigned int done_reduce;      // CTAs of the running reduce kernel that finished (rank-local)
};

struct Layout {
  size_t xin, ids, probs, pin, bytes;  // byte offsets in the slab
};

__host__ __device__ inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

__host__ __device__ inline Layout slab_layout(int N, int T, int H, int K) {
  Layout L;
  size_t off = align256(sizeof(Control));
  const size_t rows = (size_t)2 * N * T;  // [parity][rank][token]
  L.xin = off;
  off += align256(rows * H * 4);
  L.ids = off;
  off += align256(rows * K * 4);
  L.probs = off;
  off += align256(rows * K * 4);
  L.pin = off;
  off += align256(rows * H * 4);
  L.bytes = off;
  return L;
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 waits until every rank's counter in `cnt` reaches `target`;
// false (and a recorded timeout) if one does not within the limit.
__device__ bool wait_counts(const unsigned int* cnt, int N, unsigned int target, int* err) {
  for (int r = 0; r < N; ++r) {
    uint32_t i = 0;
    while (load_acquire_sys(cnt + r) < target) {
      if (++i >= kSpinLimit) {
        set_error(err, kDevTimeout);
        return false;
      }
      if (i > 64) __nanosleep(64);
    }
  }
  return true;
}

// Called by every CTA of a push kernel after its stores: the last CTA to
// finish makes all of them visible system-wide and raises counter
// `which` (0 dispatch, 1 combine) at index `rank` in every rank's slab.
__device__ void push_done(Control* mine, uint8_t* const* slabs, int rank, int N, int which) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const unsigned int n = gridDim.x * gridDim.y;
  const unsigned int prev = atomicAdd(&mine->done_push, 1u);
  if (prev != n - 1) return;
  mine->done_push = 0;
  __threadfence_system();
  for (int q = 0; q < N; ++q) {
    Control* c = reinterpret_cast<Control*>(slabs[q]);
    atomicAdd_system(which == 0 ? &c->disp[rank] : &c->comb[rank], 1u);
  }
}

// grid (blocks, N): y = destination rank q.  Rows of x [T][H] and the ids /
// probs [T][K] go to slot `rank` of q's receive areas (parity of the step).
__global__ void dispatch_push_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                                     const float4* __restrict__ x, const int32_t* __restrict__ ids,
                                     const float* __restrict__ probs) {
  const int q = blockIdx.y;
  Control* mine = reinterpret_cast<Control*>(slabs[rank]);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int par = mine->step & 1u;
  uint8_t* dst = slabs[q];
  const size_t slot = ((size_t)par * N + rank) * T;  // first row of the slot
  float4* xd = reinterpret_cast<float4*>(dst + L.xin) + slot * (H / 4);
  const size_t n4 = (size_t)T * (H / 4);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    xd[i] = x[i];
  if (blockIdx.x == 0) {
    int32_t* idd = reinterpret_cast<int32_t*>(dst + L.ids) + slot * K;
    float* pd = reinterpret_cast<float*>(dst + L.probs) + slot * K;
    for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
      idd[i] = ids[i];
      pd[i] = probs[i];
    }
  }
  push_done(mine, slabs, rank, N, 0);
}

// Waits for all N dispatch pushes of this step, then copies the receive
// slots into the contiguous buffers x_all [N*T][H], ids_all / probs_all
// [N*T][K] (rank order).
__global__ void dispatch_gather_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                                       float4* __restrict__ x_all, int32_t* __restrict__ ids_all,
                                       float* __restrict__ probs_all, int* __restrict__ err) {
  __shared__ int ok;
  uint8_t* mine_b = slabs[rank];
  Control* mine = reinterpret_cast<Control*>(mine_b);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int step = mine->step, par = step & 1u;
  if (threadIdx.x == 0) ok = wait_counts(mine->disp, N, step + 1, err) ? 1 : 0;
  __syncthreads();
  if (!ok) return;
  const size_t base = (size_t)par * N * T;
  const float4* xs = reinterpret_cast<const float4*>(mine_b + L.xin) + base * (H / 4);
  const size_t n4 = (size_t)N * T * (H / 4);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    x_all[i] = xs[i];
  const int32_t* is = reinterpret_cast<const int32_t*>(mine_b + L.ids) + base * K;
  const float* ps = reinterpret_cast<const float*>(mine_b + L.probs) + base * K;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)N * T * K;
       i += (size_t)gridDim.x * blockDim.x) {
    ids_all[i] = is[i];
    probs_all[i] = ps[i];
  }
}

// grid (blocks, N): y = home rank q of the tokens.  Rows [q*T, (q+1)*T) of
// partial [N*T][H] go to slot `rank` of q's partial area.
__global__ void combine_push_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                                    const float4* __restrict__ partial) {
  const int q = blockIdx.y;
  Control* mine = reinterpret_cast<Control*>(slabs[rank]);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int par = mine->step & 1u;
  float4* pd = reinterpret_cast<float4*>(slabs[q] + L.pin) + ((size_t)par * N + rank) * T * (H / 4);
  const float4* ps = partial + (size_t)q * T * (H / 4);
  const size_t n4 = (size_t)T * (H / 4);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    pd[i] = ps[i];
  push_done(mine, slabs, rank, N, 1);
}

// Waits for the N partials of this step's home tokens and sums them in
// rank order; the last CTA to finish advances the step count.
__global__ void combine_reduce_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                                      float4* __restrict__ out, int* __restrict__ err) {
  __shared__ int ok;
  uint8_t* mine_b = slabs[rank];
  Control* mine = reinterpret_cast<Control*>(mine_b);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int step = mine->step, par = step & 1u;
  if (threadIdx.x == 0) ok = wait_counts(mine->comb, N, step + 1, err) ? 1 : 0;
  __syncthreads();
  if (ok) {
    const size_t n4 = (size_t)T * (H / 4);
    const float4* pin = reinterpret_cast<const float4*>(mine_b + L.pin) + (size_t)par * N * n4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
      float4 o = pin[i];
      for (int r = 1; r < N; ++r) {
        const float4 v = pin[(size_t)r * n4 + i];
        o.x = __fadd_rn(o.x, v.x);
        o.y = __fadd_rn(o.y, v.y);
        o.z = __fadd_rn(o.z, v.z);
        o.w = __fadd_rn(o.w, v.w);
      }
      out[i] = o;
    }
  }
  // Every CTA has read the step count; the last one advances it.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int n = gridDim.x;
    if (atomicAdd(&mine->done_reduce, 1u) == n - 1) {
      mine->done_reduce = 0;
      mine->step = step + 1;
      __threadfence();
    }
  }
}

int grid_blocks(size_t n4) {
  size_t g = (n4 + 255) / 256;
  if (g > 148 * 4) g = 148 * 4;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace ep
}  // namespace mrml

using namespace mrml::ep;

namespace {

int ep_args_ok(void* const* slabs, int rank, int N, int T, int H, int K) {
  if (!slabs || N < 1 || N > kMaxRanks || rank < 0 || rank >= N || T < 1 || H < 4 || H % 4 != 0 || K < 1 || K > 64)
    return MRML_ERR_INVALID_ARGUMENT;
  return MRML_OK;
}

int launched() { return cudaPeekAtLastError() == cudaSuccess ? MRML_OK : MRML_ERR_CUDA; }

}  // namespace

extern "C" {

size_t mrml_moe_ep_slab_bytes(int N, int T, int H, int K) {
  if (N < 1 || N > kMaxRanks || T < 1 || H < 4 || H % 4 != 0 || K < 1 || K > 64) return 0;
  return slab_layout(N, T, H, K).bytes;
}

int mrml_moe_ep_slab_alloc(size_t bytes, void** slab) {
  if (!slab || bytes < sizeof(Control)) return MRML_ERR_INVALID_ARGUMENT;
  *slab = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MRML_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return MRML_ERR_CUDA;
  }
  *slab = p;
  return MRML_OK;
}

int mrml_moe_ep_slab_free(void* slab) {
  if (!slab) return MRML_OK;
  return cudaFree(slab) == cudaSuccess ? MRML_OK : MRML_ERR_CUDA;
}

int mrml_moe_ipc_get_handle(const void* slab, void* handle) {
  if (!slab || !handle) return MRML_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(slab)) != cudaSuccess) return MRML_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return MRML_OK;
}

int mrml_moe_ipc_open_handle(const void* handle, void** slab) {
  if (!handle || !slab) return MRML_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *slab = nullptr;
  if (cudaIpcOpenMemHandle(slab, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MRML_ERR_CUDA;
  return MRML_OK;
}

int mrml_moe_ipc_close_handle(void* slab) {
  if (!slab) return MRML_OK;
  return cudaIpcCloseMemHandle(slab) == cudaSuccess ? MRML_OK : MRML_ERR_CUDA;
}

int mrml_moe_ep_dispatch(void* const* slabs, int rank, int N, int T, int H, int K, const float* x, const int32_t* ids,
                         const float* probs, float* x_all, int32_t* ids_all, float* probs_all, int* status,
                         mrml_stream_t stream) {
  int st = ep_args_ok(slabs, rank, N, T, H, K);
  if (st != MRML_OK) return st;
  if (!x || !ids || !probs || !x_all || !ids_all || !probs_all || !status) return MRML_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)x | (uintptr_t)x_all) & 15) != 0) return MRML_ERR_INVALID_ARGUMENT;
  const cudaStream_t s = (cudaStream_t)stream;
  uint8_t* const* sl = reinterpret_cast<uint8_t* const*>(slabs);
  const size_t n4 = (size_t)T * (H / 4);
  dispatch_push_kernel<<<dim3(grid_blocks(n4), N), 256, 0, s>>>(sl, rank, N, T, H, K,
                                                               reinterpret_cast<const float4*>(x), ids, probs);
  if ((st = launched()) != MRML_OK) return st;
  dispatch_gather_kernel<<<grid_blocks(n4 * N), 256, 0, s>>>(sl, rank, N, T, H, K, reinterpret_cast<float4*>(x_all),
                                                             ids_all, probs_all, status);
  return launched();
}

int mrml_moe_ep_combine(void* const* slabs, int rank, int N, int T, int H, int K, const float* partial, float* out,
                        int* status, mrml_stream_t stream) {
  int st = ep_args_ok(slabs, rank, N, T, H, K);
  if (st != MRML_OK) return st;
  if (!partial || !out || !status) return MRML_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)partial | (uintptr_t)out) & 15) != 0) return MRML_ERR_INVALID_ARGUMENT;
  const cudaStream_t s = (cudaStream_t)stream;
  uint8_t* const* sl = reinterpret_cast<uint8_t* const*>(slabs);
  const size_t n4 = (size_t)T * (H / 4);
  combine_push_kernel<<<dim3(grid_blocks(n4), N), 256, 0, s>>>(sl, rank, N, T, H, K,
                                                              reinterpret_cast<const float4*>(partial));
  if ((st = launched()) != MRML_OK) return st;
  combine_reduce_kernel<<<grid_blocks(n4), 256, 0, s>>>(sl, rank, N, T, H, K, reinterpret_cast<float4*>(out), status);
  return launched();
}

}  // extern "C"
