// ep_p2p.cu — the expert-parallel exchange over NVLink peer memory.
//
// The expert-parallel layer (rank r of N holds experts [r*E/N, (r+1)*E/N)
// and T home tokens) needs two exchanges per step.  Both are sparse: a token
// goes only to the ranks that own one of its experts, and only those ranks
// send a partial output back.  The library's kernels write straight into the
// other GPUs' memory (CUDA IPC mappings of each rank's "slab"), without a
// collective library:
//
//   dispatch (home rank):   quantise each home row to Q8_0 once (the layer's
//     own activation quantiser, quant.rs:193-228), store its values and f16
//     scales into every rank that owns one of its experts, store the ids and
//     weights of all home tokens into every rank, then raise a counter in
//     every rank's slab (system-scope atomics);
//   receive (expert rank):  wait until all N counters show this step, copy
//     the N ranks' ids / weights into the workspace; the expert kernels then
//     read the received Q8_0 rows straight from the slab;
//   combine push (expert rank): per received token with a pair here, the
//     slot-ordered partial sum over this rank's pairs (the single-device
//     combine's arithmetic) is stored into the token's home rank, then a
//     counter is raised in every rank's slab;
//   reduce (home rank):     wait for all N combine pushes, then sum each home
//     token's partials over the ranks that own its experts, in rank order.
//
// Slab layout (identical on every rank, offsets from slab_layout): control
// counters written by peers, rank-local counters, and double-buffered
// receive areas indexed by the parity of the rank's step count.  Counters
// only grow (each source adds 1 per step), so no reset is needed and a step
// waits for "count >= step + 1".  The step count lives in device memory and
// every kernel reads it, so a captured step replays correctly.  Double
// buffering makes slot reuse safe: a rank writes parity p of a peer's areas
// in step s + 2 only after it has waited, in step s + 1, for that peer's
// push of step s + 1, which the peer issues after it finished reading
// parity p in step s (dispatch areas: the peer's combine push follows its
// expert kernels; combine areas: the peer's dispatch push follows its
// reduce).
//
// Every wait is bounded (a spin limit, kSpinLimit polls by default); a wait
// that gives up records MRML_ERR_DEVICE_TIMEOUT in the caller's status word
// and the kernel leaves without touching the data it would have produced, so
// a rank that stops never hangs the others' GPUs.
#include <string.h>

#include <atomic>

#include "../../include/mrml_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace mrml {
namespace ep {

struct Control {
  unsigned int disp[kEpMaxRanks];  // dispatch pushes received from each rank
  unsigned int comb[kEpMaxRanks];  // combine pushes received from each rank
  unsigned int step;               // steps completed by this rank (rank-local)
  unsigned int done_push;          // CTAs of the running push kernel that finished (rank-local)
  unsigned int done_reduce;        // CTAs of the running reduce kernel that finished (rank-local)
};

struct Layout {
  size_t ids, probs, q, d, part, bytes;  // byte offsets in the slab
};

__host__ __device__ inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Receive areas, each [parity][source rank][token]: ids / probs [K] of every
// home token of the source; the Q8_0 values [H] and f16 scales [H/32] of
// the source's tokens that have a pair here; the partial rows [H] of this
// rank's home tokens computed by the source.
__host__ __device__ inline Layout slab_layout(int N, int T, int H, int K) {
  Layout L;
  size_t off = align256(sizeof(Control));
  const size_t rows = (size_t)2 * N * T;
  L.ids = off;
  off += align256(rows * K * 4);
  L.probs = off;
  off += align256(rows * K * 4);
  L.q = off;
  off += align256(rows * H);
  L.d = off;
  off += align256(rows * (H / 32) * 2);
  L.part = off;
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
// false (and a recorded timeout) if one does not within `limit` polls.
__device__ bool wait_counts(const unsigned int* cnt, int N, unsigned int target, unsigned int limit, int* err) {
  for (int r = 0; r < N; ++r) {
    uint32_t i = 0;
    while (load_acquire_sys(cnt + r) < target) {
      if (++i >= limit) {
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

// Ranks that own one of token t's experts (pairs with alpha > 1e-4 and an
// id in [0, E); experts [q*E/N, (q+1)*E/N) on rank q), as a bit mask;
// every lane of the warp gets it.
__device__ __forceinline__ unsigned int owner_mask(const int32_t* __restrict__ ids, const float* __restrict__ probs,
                                                   int t, int K, int E, int N) {
  const int lane = threadIdx.x & 31, per = E / N;
  unsigned int m = 0;
  for (int k = lane; k < K; k += 32) {
    const int id = ids[(size_t)t * K + k];
    if (probs[(size_t)t * K + k] > 0.0001f && id >= 0 && id < E) m |= 1u << (id / per);
  }
  return __reduce_or_sync(0xffffffffu, m);
}

// Dispatch push.  One warp per (home token, 128-element chunk of 4 quant
// blocks): lane l holds elements [4l, 4l+4) of the chunk, so block l / 8 is
// quantised to Q8_0 by 8 lanes (quant.rs:193-228, as quantize_rows_kernel
// does) and the chunk's 128 value bytes leave as one coalesced 128-byte
// store per destination: every rank that owns one of the token's experts.
// Threads [0, T*K) of the grid also store the ids and weights of all home
// tokens into every rank.
__global__ void dispatch_push_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int E, int K,
                                     const float* __restrict__ x, const int32_t* __restrict__ ids,
                                     const float* __restrict__ probs) {
  Control* mine = reinterpret_cast<Control*>(slabs[rank]);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int par = mine->step & 1u;
  const int lane = threadIdx.x & 31, nb = H / 32, nch = (nb + 3) / 4;
  const size_t slot = ((size_t)par * N + rank) * T;  // first row of this rank's slot
  const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gtid < (long long)T * K) {
    const int32_t id = ids[gtid];
    const float p = probs[gtid];
    for (int q = 0; q < N; ++q) {
      reinterpret_cast<int32_t*>(slabs[q] + L.ids)[slot * K + gtid] = id;
      reinterpret_cast<float*>(slabs[q] + L.probs)[slot * K + gtid] = p;
    }
  }
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < (long long)T * nch;
       w += warps) {
    const int t = (int)(w / nch), c = (int)(w % nch);
    const unsigned int mask = owner_mask(ids, probs, t, K, E, N);
    if (mask == 0) continue;  // warp-uniform
    const int b = 4 * c + (lane >> 3);  // this lane's quant block
    const bool in = b < nb;             // uniform over the block's 8 lanes
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (in) v = *reinterpret_cast<const float4*>(x + (size_t)t * H + 128 * c + 4 * (lane & 31));
    const float e[4] = {v.x, v.y, v.z, v.w};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = fabsf(e[i]);
      amax = fmaxf(amax, a > 0.f ? a : 0.f);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = __fdiv_rn(amax, 127.0f);
    const uint32_t d16 = f32_to_f16_trunc(scale);
    const float inv = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = round_half_away(__fmul_rn(e[i], inv));
      if (r != r) r = 0.f;
      r = fminf(fmaxf(r, -128.f), 127.f);
      word |= ((uint32_t)(int)r & 0xffu) << (8 * i);
    }
    for (int q = 0; q < N; ++q) {
      if (!(mask >> q & 1u) || !in) continue;
      reinterpret_cast<uint32_t*>(slabs[q] + L.q + (slot + t) * H + 128 * c)[lane] = word;
      if ((lane & 7) == 0) reinterpret_cast<uint16_t*>(slabs[q] + L.d)[(slot + t) * nb + b] = (uint16_t)d16;
    }
  }
  push_done(mine, slabs, rank, N, 0);
}

// Receive: waits for all N dispatch pushes of this step, then copies the N
// ranks' ids / weights into ids_all / probs_all [N*T][K] (rank order) and
// (CTA 0) publishes the step's received Q8_0 rows: rows[0] = values
// [N*T][H], rows[1] = f16 scales [N*T][H/32].  After a timeout the copies
// are zero weights, so that the expert kernels that follow find no pairs.
__global__ void recv_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                            int32_t* __restrict__ ids_all, float* __restrict__ probs_all,
                            const uint8_t** __restrict__ rows, unsigned int limit, int* __restrict__ err) {
  __shared__ int ok;
  uint8_t* mine_b = slabs[rank];
  Control* mine = reinterpret_cast<Control*>(mine_b);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int step = mine->step, par = step & 1u;
  if (threadIdx.x == 0) ok = wait_counts(mine->disp, N, step + 1, limit, err) ? 1 : 0;
  __syncthreads();
  const size_t base = (size_t)par * N * T;
  const int32_t* is = reinterpret_cast<const int32_t*>(mine_b + L.ids) + base * K;
  const float* ps = reinterpret_cast<const float*>(mine_b + L.probs) + base * K;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)N * T * K;
       i += (size_t)gridDim.x * blockDim.x) {
    ids_all[i] = ok ? is[i] : 0;
    probs_all[i] = ok ? ps[i] : 0.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    rows[0] = mine_b + L.q + base * H;
    rows[1] = mine_b + L.d + base * (H / 32) * 2;
  }
  pdl_trigger();
}

// The decode kernel's group-major operand from the received Q8_0 rows (as
// gather_groups_kernel does from quantize_rows_kernel's output): one warp per
// (position group, block); lane (j = lane / 4, part = lane % 4) copies 8
// bytes of position j's row.  The block's value sum (the Q4_0 correction)
// is summed over the row's 32 bytes.  Positions in use: *poff_end.
__global__ void recv_gather_kernel(const uint8_t* const* __restrict__ rows, const int32_t* __restrict__ pair_at,
                                   const int32_t* __restrict__ poff_end, int H, int K, int wq4, int npad,
                                   int8_t* __restrict__ bq, int2* __restrict__ bsc) {
  pdl_wait();
  pdl_trigger();
  const int nb = H / 32;
  const int8_t* xq = reinterpret_cast<const int8_t*>(rows[0]);
  const uint16_t* xd = reinterpret_cast<const uint16_t*>(rows[1]);
  const long long total = (long long)(*poff_end / 8) * nb;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31, j = lane >> 2, part = lane & 3;
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
    const int g = (int)(w / nb), b = (int)(w % nb);
    const int pos = 8 * g + j;
    const int pair = pair_at[pos];
    const int t = pair >= 0 ? pair / K : -1;
    uint2 v = make_uint2(0u, 0u);
    if (t >= 0) v = *reinterpret_cast<const uint2*>(xq + (size_t)t * H + 32 * b + 8 * part);
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) s += (int)(int8_t)(v.x >> (8 * k)) + (int)(int8_t)(v.y >> (8 * k));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    uint8_t* dst = reinterpret_cast<uint8_t*>(bq) + act_group_offset(true, b, g, nb, npad) + (part >> 1) * 128 +
                   j * 16 + 8 * (part & 1);
    *reinterpret_cast<uint2*>(dst) = v;
    if (part == 0) {
      float d = 0.f;
      int corr = kMagicI;
      if (t >= 0) {
        d = f16_bits_to_f32(xd[(size_t)t * nb + b]);
        if (wq4) corr = kMagicI - 8 * s;
      }
      store_act_scale_gm(bsc, b, pos, nb, d, corr);
    }
  }
}

// Combine push.  CTAs (x, c) walk the received token slots j = src * T + t
// (j = x, x + gridDim.x, ...) over chunk c of kCombThreads float4 columns: if
// this rank computed any of the token's pairs, each thread forms its 4
// columns of the slot-ordered partial (sum over k ascending of (alpha_k *
// ydown[pos]) * scale[id], from 0; the single-device combine's arithmetic,
// model.rs:2163-2165) and stores them into rank src's partial area.  A
// bounded grid keeps the per-CTA system-scope release of push_done rare.
constexpr int kCombThreads = 128;

__global__ void __launch_bounds__(kCombThreads)
    combine_push_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int K,
                        const float* __restrict__ ydown, const int32_t* __restrict__ pos,
                        const int32_t* __restrict__ ids_all, const float* __restrict__ probs_all,
                        const float* __restrict__ down_scale) {
  __shared__ int s_pos[kMaxTopK];
  __shared__ float s_alpha[kMaxTopK], s_sc[kMaxTopK];
  __shared__ int s_n;
  pdl_wait();
  Control* mine = reinterpret_cast<Control*>(slabs[rank]);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int par = mine->step & 1u;
  const int i4 = blockIdx.y * kCombThreads + threadIdx.x;
  for (long long j = blockIdx.x; j < (long long)N * T; j += gridDim.x) {
    // the token's pairs here, in slot order
    if (threadIdx.x < 32) {
      int n = 0;
      for (int k0 = 0; k0 < K; k0 += 32) {
        const int k = k0 + (int)threadIdx.x;
        const int p = k < K ? pos[j * K + k] : -1;
        const unsigned int bal = __ballot_sync(0xffffffffu, p >= 0);
        if (p >= 0) {
          const int at = n + __popc(bal & ((1u << threadIdx.x) - 1u));
          s_pos[at] = p;
          s_alpha[at] = probs_all[j * K + k];
          s_sc[at] = down_scale ? down_scale[ids_all[j * K + k]] : 1.0f;
        }
        n += __popc(bal);
      }
      if (threadIdx.x == 0) s_n = n;
    }
    __syncthreads();
    const int n = s_n;
    if (n > 0 && i4 < H / 4) {
      const int src = (int)(j / T), t = (int)(j % T);
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k0 = 0; k0 < n; k0 += 4) {
        float4 y[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (k0 + u < n) y[u] = reinterpret_cast<const float4*>(ydown + (size_t)s_pos[k0 + u] * H)[i4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (k0 + u >= n) break;
          const float a = s_alpha[k0 + u], sc = s_sc[k0 + u];
          o.x = __fadd_rn(o.x, __fmul_rn(__fmul_rn(a, y[u].x), sc));
          o.y = __fadd_rn(o.y, __fmul_rn(__fmul_rn(a, y[u].y), sc));
          o.z = __fadd_rn(o.z, __fmul_rn(__fmul_rn(a, y[u].z), sc));
          o.w = __fadd_rn(o.w, __fmul_rn(__fmul_rn(a, y[u].w), sc));
        }
      }
      float4* dst = reinterpret_cast<float4*>(slabs[src] + L.part) + (((size_t)par * N + rank) * T + t) * (H / 4);
      dst[i4] = o;
    }
    __syncthreads();  // the slot list is rebuilt for the next token
  }
  push_done(mine, slabs, rank, N, 1);
}

// Reduce: waits for the N combine pushes of this step, then out[t] = the
// partials of the ranks that own one of t's experts, summed in rank order
// (0 for a token with no pair); the last CTA to finish advances the step.
// CTAs (x, c) walk the home tokens t = x, x + gridDim.x, ... over chunk c of
// float4 columns.  After a timeout `out` is left untouched.
__global__ void __launch_bounds__(kCombThreads)
    combine_reduce_kernel(uint8_t* const* __restrict__ slabs, int rank, int N, int T, int H, int E, int K,
                          const int32_t* __restrict__ ids, const float* __restrict__ probs, float4* __restrict__ out,
                          unsigned int limit, int* __restrict__ err) {
  __shared__ int ok;
  __shared__ unsigned int s_mask;
  uint8_t* mine_b = slabs[rank];
  Control* mine = reinterpret_cast<Control*>(mine_b);
  const Layout L = slab_layout(N, T, H, K);
  const unsigned int step = mine->step, par = step & 1u;
  if (threadIdx.x == 0) ok = wait_counts(mine->comb, N, step + 1, limit, err) ? 1 : 0;
  __syncthreads();
  const int i4 = blockIdx.y * kCombThreads + threadIdx.x;
  const float4* part = reinterpret_cast<const float4*>(mine_b + L.part) + (size_t)par * N * T * (H / 4);
  for (int t = blockIdx.x; ok && t < T; t += gridDim.x) {
    if (threadIdx.x < 32) {
      const unsigned int m = owner_mask(ids, probs, t, K, E, N);
      if (threadIdx.x == 0) s_mask = m;
    }
    __syncthreads();
    const unsigned int mask = s_mask;
    if (i4 < H / 4) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      bool first = true;
      for (int q = 0; q < N; ++q) {
        if (!(mask >> q & 1u)) continue;
        const float4 v = part[((size_t)q * T + t) * (H / 4) + i4];
        if (first) {
          o = v;
          first = false;
        } else {
          o.x = __fadd_rn(o.x, v.x);
          o.y = __fadd_rn(o.y, v.y);
          o.z = __fadd_rn(o.z, v.z);
          o.w = __fadd_rn(o.w, v.w);
        }
      }
      out[(size_t)t * (H / 4) + i4] = o;
    }
    __syncthreads();  // s_mask is rewritten for the next token
  }
  // Every CTA has read the step count; the last one advances it.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int n = gridDim.x * gridDim.y;
    if (atomicAdd(&mine->done_reduce, 1u) == n - 1) {
      mine->done_reduce = 0;
      mine->step = step + 1;
      __threadfence();
    }
  }
}

int grid_for(long long items, int per_cta) {
  long long g = (items + per_cta - 1) / per_cta;
  if (g > 148 * 8) g = 148 * 8;
  return (int)(g < 1 ? 1 : g);
}

std::atomic<unsigned int> g_spin_limit{kSpinLimit};

}  // namespace ep

size_t ep_slab_bytes(int N, int T, int H, int K) { return ep::slab_layout(N, T, H, K).bytes; }

void ep_set_spin_limit(unsigned int limit) { ep::g_spin_limit.store(limit ? limit : kSpinLimit); }

cudaError_t launch_ep_dispatch(uint8_t* const* slabs, int rank, int N, int T, int H, int E, int K, const float* x,
                               const int32_t* ids, const float* probs, cudaStream_t s) {
  const long long warps = (long long)T * ((H / 32 + 3) / 4);
  const int grid = std::max(ep::grid_for(warps, 8), ep::grid_for((long long)T * K, 256));
  ep::dispatch_push_kernel<<<grid, 256, 0, s>>>(slabs, rank, N, T, H, E, K, x, ids, probs);
  return cudaPeekAtLastError();
}

cudaError_t launch_ep_recv(uint8_t* const* slabs, int rank, int N, int T, int H, int K, int32_t* ids_all,
                           float* probs_all, const uint8_t** rows, int* err, cudaStream_t s) {
  const int grid = ep::grid_for((long long)N * T * K, 256 * 4);
  ep::recv_kernel<<<grid, 256, 0, s>>>(slabs, rank, N, T, H, K, ids_all, probs_all, rows,
                                       ep::g_spin_limit.load(), err);
  return cudaPeekAtLastError();
}

cudaError_t launch_ep_gather(int wtype, const uint8_t* const* rows, const int32_t* pair_at, const int32_t* poff_end,
                             int H, int K, int npad, int8_t* bq, int2* bsc, cudaStream_t s) {
  const long long warps = (long long)(npad / 8) * (H / 32);  // upper bound; the kernel reads the count
  return launch_pdl(ep::recv_gather_kernel, dim3(ep::grid_for(warps, 8)), dim3(256), 0, s, rows, pair_at, poff_end,
                    H, K, wtype == kQ4_0 ? 1 : 0, npad, bq, bsc);
}

cudaError_t launch_ep_combine_push(uint8_t* const* slabs, int rank, int N, int T, int H, int K, const float* ydown,
                                   const int32_t* pos, const int32_t* ids_all, const float* probs_all,
                                   const float* down_scale, cudaStream_t s) {
  const int ny = (H / 4 + ep::kCombThreads - 1) / ep::kCombThreads;
  const int nx = (int)std::min<long long>((long long)N * T, std::max(1, 148 * 8 / ny));
  return launch_pdl(ep::combine_push_kernel, dim3((unsigned)nx, (unsigned)ny), dim3(ep::kCombThreads), 0, s, slabs,
                    rank, N, T, H, K, ydown, pos, ids_all, probs_all, down_scale);
}

cudaError_t launch_ep_reduce(uint8_t* const* slabs, int rank, int N, int T, int H, int E, int K, const int32_t* ids,
                             const float* probs, float* out, int* err, cudaStream_t s) {
  const int ny = (H / 4 + ep::kCombThreads - 1) / ep::kCombThreads;
  const dim3 grid((unsigned)std::min(T, std::max(1, 148 * 8 / ny)), (unsigned)ny);
  ep::combine_reduce_kernel<<<grid, ep::kCombThreads, 0, s>>>(slabs, rank, N, T, H, E, K, ids, probs,
                                                               reinterpret_cast<float4*>(out),
                                                               ep::g_spin_limit.load(), err);
  return cudaPeekAtLastError();
}

}  // namespace mrml

using namespace mrml::ep;

extern "C" {

size_t mrml_moe_ep_slab_bytes(int N, int T, int H, int K) {
  if (N < 1 || N > mrml::kEpMaxRanks || T < 1 || H < 32 || H % 32 != 0 || K < 1 || K > mrml::kMaxTopK) return 0;
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

}  // extern "C"
