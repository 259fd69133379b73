// router.cu — router logits, top-k and softmax for the MRML MoE layer.
//
// Reference behaviour (crates/mrml-tensor/src/model.rs:1804-1829): each logit
// is a sequential f32 dot product, x[i]*W[e,i] rounded, then added in index
// order; experts are sorted by logit descending (ties: lower expert id), the
// first K are kept and p_k = expf(l_k - l_0) / max(sum_k, 1e-6).
//
// A sequential 2816-term f32 chain per (token, expert) is latency bound
// (~6 us), so the GPU computes every logit in parallel and, with it, a
// rigorous bound B on |reference value - our value|.  The top-K choice and
// order are accepted only when every comparison that decides them is
// separated by more than the two bounds.  The few experts whose intervals
// overlap are then recomputed with the exact sequential chain, so the chosen
// ids and their order always equal the reference's.
//
// Error bound.  For the sequential sum s^_n of the rounded products the
// first-order bound is |s^_n - s_n| <= u*(sum_i |p_i| + sum_k |s^_k|), u =
// 2^-24, and sum_k |s^_k| <= sum_k |s_k| + n*gamma_n*sum|p_i|.  Lane l of a
// warp sums a contiguous chunk c of the row in f32; sum_k |s_k| over the
// chunk is at most len_c*|S_c| + sum_{k in c} |r_k|, where S_c is the exact
// prefix before the chunk (scanned in double from the chunk sums) and r_k the
// lane's running sum.  Our own value carries at most u*(sum|p| + sum|r_k|).
#include "common.cuh"
#include "kernels.h"

namespace mrml {

constexpr int kRouterWarps = 8;
constexpr int kMaxCandidates = 64;  // also the largest supported K
constexpr int kTopkWarps = 8;       // tokens per top-k CTA
constexpr int kExactRows = 4;       // flagged expert rows staged per pass

// Row pitch (floats) of the chunked layout: lane l owns elements
// [l*C, l*C + C) of a row, stored at l*pitch; an odd pitch keeps the 32
// lanes' reads of one chunk offset on 32 different banks.
__host__ __device__ inline int chunk_len(int H) { return (H + 31) / 32; }
__host__ __device__ inline int chunk_pitch(int H) { return chunk_len(H) | 1; }

// Copies `rows` rows of length H (row stride H) into the chunked layout.
// Each thread loads a batch of elements into registers before storing them,
// so that the global loads of a batch are in flight together; the chunk
// index and offset of element i advance incrementally.
__device__ __forceinline__ void stage_chunked(float* dst, const float* __restrict__ src, int rows, int H) {
  constexpr int kBatch = 16;
  const int C = chunk_len(H), pitch = chunk_pitch(H), row_floats = 32 * pitch;
  const int step = blockDim.x, dq = step / C, dr = step % C;
  for (int r = 0; r < rows; ++r) {
    const float* s = src + (size_t)r * H;
    float* d = dst + r * row_floats;
    int q = threadIdx.x / C, rem = threadIdx.x % C;
    for (int i0 = threadIdx.x; i0 < H; i0 += step * kBatch) {
      float v[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int i = i0 + k * step;
        v[k] = i < H ? s[i] : 0.f;
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        if (i0 + k * step < H) d[q * pitch + rem] = v[k];
        q += dq;
        rem += dr;
        if (rem >= C) {
          rem -= C;
          ++q;
        }
      }
    }
  }
}

// grid (ceil(E / epc), ceil(T / tpc)), block 32*kRouterWarps.  The CTA
// stages tpc token rows of x and epc expert rows of W in shared memory,
// then one warp per (token, expert) pair computes the logit and its error
// bound; lane l owns the contiguous chunk [l*C, l*C + C) of the row.
// With `bulk` (H % 128 == 0, 16-byte aligned rows) each row arrives by one
// bulk copy into a dense layout (row pitch H) and lanes read float4s: the
// 8 lanes of a quarter-warp then hit at most 2 requests per bank group.
// Otherwise rows are staged by coalesced loads into a padded chunk layout.
// Writes logits[t*E + e] and bounds[t*E + e].
__global__ void __launch_bounds__(32 * kRouterWarps)
    router_logits_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                         float* __restrict__ bounds, int H, int E, int T, int epc, int tpc, int bulk,
                         int* __restrict__ err) {
  extern __shared__ __align__(16) float rsm[];
  __shared__ __align__(8) uint64_t bar;
  const int C = chunk_len(H);
  const int pitch = bulk ? C : chunk_pitch(H);  // lane chunk stride
  const int row_floats = bulk ? H : 32 * pitch;
  const int e0 = blockIdx.x * epc, t0 = blockIdx.y * tpc;
  const int ne = min(epc, E - e0), nt = min(tpc, T - t0);
  float* xs = rsm;                     // [tpc][row_floats]
  float* ws = rsm + tpc * row_floats;  // [epc][row_floats]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_init(&bar, 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&bar, (uint32_t)((nt + ne) * H * 4));
      for (int r = 0; r < nt; ++r) bulk_g2s(xs + r * row_floats, x + (size_t)(t0 + r) * H, H * 4, &bar);
      for (int r = 0; r < ne; ++r) bulk_g2s(ws + r * row_floats, W + (size_t)(e0 + r) * H, H * 4, &bar);
    }
    if (!mbar_wait_bounded(&bar, 0, err)) return;
  } else {
    stage_chunked(xs, x + (size_t)t0 * H, nt, H);
    stage_chunked(ws, W + (size_t)e0 * H, ne, H);
    __syncthreads();
  }

  const int start = lane * C;
  const int len = max(0, min(C, H - start));
  const float u = 5.9604644775390625e-8f;  // 2^-24
  for (int p = warp; p < ne * nt; p += kRouterWarps) {
    const int el = p % ne, tl = p / ne;
    const float* xl = xs + tl * row_floats + lane * pitch;
    const float* wl = ws + el * row_floats + lane * pitch;
    float r = 0.f, A = 0.f, P = 0.f;
    if (bulk) {
      for (int j = 0; j < len; j += 4) {
        const float4 a = *reinterpret_cast<const float4*>(xl + j);
        const float4 b = *reinterpret_cast<const float4*>(wl + j);
        const float p0 = __fmul_rn(a.x, b.x), p1 = __fmul_rn(a.y, b.y);
        const float p2 = __fmul_rn(a.z, b.z), p3 = __fmul_rn(a.w, b.w);
        r = __fadd_rn(r, p0);
        A += fabsf(r);
        r = __fadd_rn(r, p1);
        A += fabsf(r);
        r = __fadd_rn(r, p2);
        A += fabsf(r);
        r = __fadd_rn(r, p3);
        A += fabsf(r);
        P += (fabsf(p0) + fabsf(p1)) + (fabsf(p2) + fabsf(p3));
      }
    } else {
#pragma unroll 4
      for (int j = 0; j < len; ++j) {
        const float prod = __fmul_rn(xl[j], wl[j]);
        r = __fadd_rn(r, prod);
        A += fabsf(r);
        P += fabsf(prod);
      }
    }
    // Exclusive prefix of the chunk sums, in double.
    double incl = (double)r;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const double excl = incl - (double)r;
    const double total = __shfl_sync(0xffffffffu, incl, 31);
    float s_part = (float)len * (float)fabs(excl) + A;
    float a_part = A;
    float p_part = P;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s_part += __shfl_xor_sync(0xffffffffu, s_part, o);
      a_part += __shfl_xor_sync(0xffffffffu, a_part, o);
      p_part += __shfl_xor_sync(0xffffffffu, p_part, o);
    }
    if (lane == 0) {
      const float center = (float)total;
      const float n = (float)H;
      const float gamma = n * u / (1.f - n * u);
      // The bound's own f32 sums carry relative errors of at most n*u; the
      // 1.01 factors cover them.
      float B = u * (2.f * p_part + s_part + a_part) * 1.01f + n * gamma * u * p_part * 1.01f;
      // Slack for rounding the center to f32 and for the f32 comparisons of
      // c - B against c' + B' made by the top-k kernel.
      B += 4.f * fabsf(center) * u + fabsf((float)(total - (double)center)) + 1e-30f;
      logits[(size_t)(t0 + tl) * E + e0 + el] = center;
      bounds[(size_t)(t0 + tl) * E + e0 + el] = B;
    }
  }
}

// (value desc, id asc) ordering used by the reference's GPU top-8
// (kernels.rs:944-968) and by the north star for exact ties.
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Warp-wide top-K of the values held by the lanes (expert lane+32m in
// val[m]); writes the chosen ids and values, best first, to cand/cval.
template <int PL>
__device__ __forceinline__ void warp_topk(const float (&val)[PL], int E, int K, int* cand, float* cval,
                                          uint32_t& taken) {
  const int lane = threadIdx.x & 31;
  taken = 0;
  for (int k = 0; k < K; ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int m = 0; m < PL; ++m) {
      const int e = lane + 32 * m;
      if (e < E && !(taken >> m & 1u) && better(val[m], e, bv, bi)) {
        bv = val[m];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == 0) {
      cand[k] = bi;
      cval[k] = bv;
    }
  }
  __syncwarp();
}

// The reference's exact value of one logit: sequential f32, mul then add,
// over rows staged in shared memory (vector loads when H % 4 == 0; the order
// of the additions is the reference's either way).
__device__ __forceinline__ float exact_logit_smem(const float* __restrict__ xs, const float* __restrict__ ws, int H) {
  float dot = 0.f;
  int i = 0;
  if ((H & 3) == 0) {
    // The chain is a dependent sequence of adds; unrolling lets the shared-
    // memory loads run ahead of it.
#pragma unroll 8
    for (; i < H; i += 4) {
      const float4 a = *reinterpret_cast<const float4*>(xs + i);
      const float4 b = *reinterpret_cast<const float4*>(ws + i);
      dot = __fadd_rn(dot, __fmul_rn(a.x, b.x));
      dot = __fadd_rn(dot, __fmul_rn(a.y, b.y));
      dot = __fadd_rn(dot, __fmul_rn(a.z, b.z));
      dot = __fadd_rn(dot, __fmul_rn(a.w, b.w));
    }
  }
  for (; i < H; ++i) dot = __fadd_rn(dot, __fmul_rn(xs[i], ws[i]));
  return dot;
}

struct TopkShared {
  int cand[kTopkWarps][kMaxCandidates];
  float cval[kTopkWarps][kMaxCandidates];
  float cbnd[kTopkWarps][kMaxCandidates];
  int flag[kTopkWarps][kMaxCandidates];
  int count[kTopkWarps];
  int pending[kTopkWarps];  // warps of this CTA whose token needs exact values
  int n_pending;
};

// Per-token selection tail: order Z (count candidates) by (value desc, id
// asc), then the reference's softmax over the first K.
__device__ void finish_token(int* cand, float* cval, int count, int K, int t, int32_t* ids, float* probs) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    for (int i = 1; i < count; ++i) {
      const float v = cval[i];
      const int c = cand[i];
      int j = i - 1;
      while (j >= 0 && better(v, c, cval[j], cand[j])) {
        cval[j + 1] = cval[j];
        cand[j + 1] = cand[j];
        --j;
      }
      cval[j + 1] = v;
      cand[j + 1] = c;
    }
  }
  __syncwarp();
  // model.rs:1819-1829: p_k = expf(l_k - l_0), summed in k order, then
  // divided by max(sum, 1e-6).  Lanes compute the exponentials in parallel;
  // lane 0 adds them in k order.
  const float max_l = cval[0];
  __syncwarp();
  for (int k = lane; k < K; k += 32) cval[k] = exp_f32(__fsub_rn(cval[k], max_l));
  __syncwarp();
  float sum = 0.f;
  if (lane == 0)
    for (int k = 0; k < K; ++k) sum = __fadd_rn(sum, cval[k]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  const float denom = sum > 1e-6f ? sum : 1e-6f;
  for (int k = lane; k < K; k += 32) {
    ids[(size_t)t * K + k] = cand[k];
    probs[(size_t)t * K + k] = __fdiv_rn(cval[k], denom);
  }
  __syncwarp();
}

// grid ceil(T / kTopkWarps), block 32*kTopkWarps; one warp per token.
// bounds == nullptr: the logits are exact inputs (route-from-logits).
// Otherwise W and x are the router weights and inputs the logits came from,
// and the dynamic shared memory (router_exact_smem(H) bytes) stages the rows
// of the exact fallback.  status[0] is the device status word, status[1]
// counts tokens that needed the fallback (status may be null without bounds).
template <int PL>
__global__ void __launch_bounds__(32 * kTopkWarps, 1)
    router_topk_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                       const float* __restrict__ bounds, int32_t* __restrict__ ids, float* __restrict__ probs, int H,
                       int E, int K, int T, int* __restrict__ status) {
  __shared__ TopkShared S;
  int* stats = status ? status + 1 : nullptr;
  extern __shared__ __align__(16) float stage[];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int t = blockIdx.x * kTopkWarps + wl;
  if (threadIdx.x == 0) S.n_pending = 0;
  __syncthreads();
  int* cand = S.cand[wl];
  float* cval = S.cval[wl];
  float* cbnd = S.cbnd[wl];
  int* flag = S.flag[wl];
  bool mine_pending = false;

  if (t < T) {
    float* lrow = logits + (size_t)t * E;
    const float* brow = bounds ? bounds + (size_t)t * E : nullptr;
    float val[PL];
    float bnd[PL];
#pragma unroll
    for (int m = 0; m < PL; ++m) {
      const int e = lane + 32 * m;
      val[m] = e < E ? lrow[e] : -INFINITY;
      bnd[m] = (e < E && brow) ? brow[e] : 0.f;
    }
    uint32_t taken;
    warp_topk<PL>(val, E, K, cand, cval, taken);
    int count = K;
    if (brow) {
      float lowest_lo = INFINITY;
#pragma unroll
      for (int m = 0; m < PL; ++m)
        if (taken >> m & 1u) lowest_lo = fminf(lowest_lo, val[m] - bnd[m]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lowest_lo = fminf(lowest_lo, __shfl_xor_sync(0xffffffffu, lowest_lo, o));
      // Bounds of the chosen experts, in the order of cand[].
      for (int k = lane; k < K; k += 32) cbnd[k] = brow[cand[k]];
      // Candidate set Z = chosen experts plus every expert whose upper bound
      // reaches lowest_lo: every other expert is below all K chosen ones in
      // the reference too, so the reference's top-K lies in Z.
#pragma unroll
      for (int m = 0; m < PL; ++m) {
        const int e = lane + 32 * m;
        const bool extra = e < E && !(taken >> m & 1u) && val[m] + bnd[m] >= lowest_lo;
        const uint32_t mask = __ballot_sync(0xffffffffu, extra);
        if (extra) {
          const int slot = count + __popc(mask & ((1u << lane) - 1u));
          if (slot < kMaxCandidates) {
            cand[slot] = e;
            cval[slot] = val[m];
            cbnd[slot] = bnd[m];
          }
        }
        count += __popc(mask);
      }
      __syncwarp();
      bool any = false;
      if (count <= kMaxCandidates) {
        for (int i = lane; i < count; i += 32) {
          const float ci = cval[i], bi_ = cbnd[i];
          bool overlap = false;
          for (int j = 0; j < count; ++j) {
            if (j == i) continue;
            const float cj = cval[j], bj = cbnd[j];
            if (!(ci - bi_ > cj + bj || cj - bj > ci + bi_)) overlap = true;
          }
          flag[i] = overlap;
          any |= overlap;
        }
      } else {
        any = true;  // bounds too wide to certify: exact values for all
      }
      mine_pending = __any_sync(0xffffffffu, any);
    }
    if (lane == 0) S.count[wl] = count;
    if (!mine_pending) finish_token(cand, cval, min(count, kMaxCandidates), K, t, ids, probs);
  }
  if (lane == 0 && mine_pending) S.pending[atomicAdd(&S.n_pending, 1)] = wl;
  __syncthreads();
  const int n_pending = S.n_pending;
  if (n_pending == 0) return;
  if (threadIdx.x == 0 && stats) atomicAdd(stats, n_pending);

  // Exact fallback, one pending token at a time: the CTA stages the token's
  // x row and up to kExactRows flagged W rows (bulk copies when rows are
  // 16-byte multiples, else coalesced loads), and one thread per row runs
  // the reference's sequential chain.
  const int pitch = (H + 3) & ~3;
  float* xs = stage;
  float* wsr = stage + pitch;
  __shared__ __align__(8) uint64_t xbar;
  const bool bulk = (H & 3) == 0 && (((uintptr_t)W | (uintptr_t)x) & 15) == 0;
  uint32_t xph = 0;
  if (threadIdx.x == 0) {
    mbar_init(&xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  for (int q = 0; q < n_pending; ++q) {
    const int w = S.pending[q];
    const int tq = blockIdx.x * kTopkWarps + w;
    float* lrow = logits + (size_t)tq * E;
    int count = S.count[w];
    const bool all = count > kMaxCandidates;
    int* qc = S.cand[w];
    float* qv = S.cval[w];
    int* qf = S.flag[w];
    const int n_items = all ? E : count;
    for (int base = 0; base < n_items; base += kExactRows) {
      __syncthreads();
      if (bulk) {
        if (threadIdx.x == 0) {
          int nrows = 0;
          for (int r = 0; r < kExactRows; ++r) {
            const int item = base + r;
            if (item < n_items && (all || qf[item])) ++nrows;
          }
          mbar_arrive_expect_tx(&xbar, (uint32_t)((base == 0 ? 1 + nrows : nrows) * H * 4));
          if (base == 0) bulk_g2s(xs, x + (size_t)tq * H, H * 4, &xbar);
          for (int r = 0; r < kExactRows; ++r) {
            const int item = base + r;
            if (item >= n_items || !(all || qf[item])) continue;
            bulk_g2s(wsr + r * pitch, W + (size_t)(all ? item : qc[item]) * H, H * 4, &xbar);
          }
        }
        if (!mbar_wait_bounded(&xbar, xph, status)) return;
        xph ^= 1;
      } else {
        if (base == 0)
          for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = x[(size_t)tq * H + i];
        for (int r = 0; r < kExactRows; ++r) {
          const int item = base + r;
          if (item >= n_items || !(all || qf[item])) continue;
          const float* wrow = W + (size_t)(all ? item : qc[item]) * H;
          for (int i = threadIdx.x; i < H; i += blockDim.x) wsr[r * pitch + i] = wrow[i];
        }
        __syncthreads();
      }
      if (threadIdx.x < kExactRows) {
        const int item = base + threadIdx.x;
        if (item < n_items && (all || qf[item])) {
          const int e = all ? item : qc[item];
          const float v = exact_logit_smem(xs, wsr + threadIdx.x * pitch, H);
          lrow[e] = v;
          if (!all) qv[item] = v;
        }
      }
    }
    __syncthreads();
    if (wl == w) {
      if (all) {
        float val[PL];
#pragma unroll
        for (int m = 0; m < PL; ++m) {
          const int e = lane + 32 * m;
          val[m] = e < E ? lrow[e] : -INFINITY;
        }
        uint32_t taken;
        warp_topk<PL>(val, E, K, qc, qv, taken);
        count = K;
      }
      finish_token(qc, qv, count, K, tq, ids, probs);
    }
  }
}

// ------------------------------------------------------------ launchers ---

// cudaFuncSetAttribute once per (kernel, device, size): it is host-side
// state and not a stream operation, but calling it on every launch costs
// host time on the decode path.
template <typename Kern>
cudaError_t ensure_smem(Kern k, size_t bytes, int* cache) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev >= 0 && dev < 16 && cache[dev] >= (int)bytes) return cudaSuccess;
  st = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (st == cudaSuccess && dev >= 0 && dev < 16) cache[dev] = (int)bytes;
  return st;
}

cudaError_t launch_router_logits(const float* W, const float* x, float* logits, float* bounds, int H, int E, int T,
                                 int* err, cudaStream_t s) {
  static int cache[16] = {0};
  const int epc = T <= 4 ? 1 : 4;
  const int tpc = T <= 4 ? T : 4;
  const dim3 grid((E + epc - 1) / epc, (T + tpc - 1) / tpc);
  const bool bulk = H % 128 == 0 && (((uintptr_t)W | (uintptr_t)x) & 15) == 0;
  const size_t smem = (size_t)(epc + tpc) * (bulk ? (size_t)H : (size_t)32 * chunk_pitch(H)) * sizeof(float);
  cudaError_t st = ensure_smem(router_logits_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  router_logits_kernel<<<grid, 32 * kRouterWarps, smem, s>>>(W, x, logits, bounds, H, E, T, epc, tpc, bulk ? 1 : 0,
                                                             err);
  return cudaPeekAtLastError();
}

size_t router_exact_smem(int H) { return (size_t)((H + 3) & ~3) * (1 + kExactRows) * sizeof(float); }

cudaError_t launch_router_topk(const float* W, const float* x, float* logits, const float* bounds, int32_t* ids,
                               float* probs, int H, int E, int K, int T, int* status, cudaStream_t s) {
  static int cache[3][16] = {{0}};
  const dim3 grid((T + kTopkWarps - 1) / kTopkWarps);
  const int block = 32 * kTopkWarps;
  const size_t smem = bounds ? router_exact_smem(H) : 0;
  cudaError_t st;
  if (E <= 32) {
    if ((st = ensure_smem(router_topk_kernel<1>, smem, cache[0])) != cudaSuccess) return st;
    router_topk_kernel<1><<<grid, block, smem, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, status);
  } else if (E <= 128) {
    if ((st = ensure_smem(router_topk_kernel<4>, smem, cache[1])) != cudaSuccess) return st;
    router_topk_kernel<4><<<grid, block, smem, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, status);
  } else {
    if ((st = ensure_smem(router_topk_kernel<8>, smem, cache[2])) != cudaSuccess) return st;
    router_topk_kernel<8><<<grid, block, smem, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, status);
  }
  return cudaPeekAtLastError();
}

}  // namespace mrml
