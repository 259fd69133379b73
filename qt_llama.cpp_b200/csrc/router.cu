// router.cu — router logits, top-k and softmax for the MRML MoE layer.
//
// Reference behaviour (crates/mrml-tensor/src/model.rs:1804-1829): each logit
// is a sequential f32 dot product, x[i]*W[e,i] rounded, then added in index
// order; experts are sorted by logit descending (ties: lower expert id), the
// first K are kept and p_k = expf(l_k - l_0) / max(sum_k, 1e-6).
//
// A sequential 2816-term f32 chain per (token, expert) is latency bound
// (~6 us), so the GPU computes every logit in parallel and, with it, a
// rigorous bound B on |CPU value - our value|.  The top-K choice and order
// are accepted only when every comparison that decides them is separated by
// more than the two bounds.  The few experts whose intervals overlap are then
// recomputed with the exact sequential chain, so the chosen ids and their
// order always equal the CPU's.
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

// grid (E, ceil(T / tokens_per_cta)), block 32*kRouterWarps.
// Writes logits[t*E + e] (our estimate) and bounds[t*E + e] (B >= 0).
__global__ void __launch_bounds__(32 * kRouterWarps)
    router_logits_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                         float* __restrict__ bounds, int H, int E, int T, int tokens_per_cta) {
  extern __shared__ float wsm[];  // 32 chunks of C floats, each padded by 1
  const int e = blockIdx.x;
  const int C = (H + 31) / 32;
  const int pitch = C + 1;
  const float* wrow = W + (size_t)e * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) wsm[(i / C) * pitch + (i % C)] = wrow[i];
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.y * tokens_per_cta;
  const int t1 = min(T, t0 + tokens_per_cta);
  const int start = lane * C;
  const int len = max(0, min(C, H - start));
  const float* wl = wsm + lane * pitch;
  const float u = 5.9604644775390625e-8f;  // 2^-24

  for (int t = t0 + warp; t < t1; t += kRouterWarps) {
    const float* xl = x + (size_t)t * H + start;
    float r = 0.f, A = 0.f, P = 0.f;
    for (int j = 0; j < len; ++j) {
      float p = __fmul_rn(xl[j], wl[j]);
      r = __fadd_rn(r, p);
      A += fabsf(r);
      P += fabsf(p);
    }
    // Exclusive prefix of the chunk sums, in double.
    double incl = (double)r;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      double v = __shfl_up_sync(0xffffffffu, incl, o);
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
      float B = u * (2.f * p_part + s_part + a_part) * 1.01f + n * gamma * u * p_part * 1.01f;
      // Slack for rounding the center to f32 and for the f32 comparisons of
      // c - B against c' + B' made by the top-k kernel.
      B += 4.f * fabsf(center) * u + fabsf((float)(total - (double)center)) + 1e-30f;
      logits[(size_t)t * E + e] = center;
      bounds[(size_t)t * E + e] = B;
    }
  }
}

// The reference's exact value of one logit: sequential f32, mul then add.
__device__ float exact_logit(const float* __restrict__ x, const float* __restrict__ w, int H) {
  float dot = 0.f;
#pragma unroll 8
  for (int i = 0; i < H; ++i) dot = __fadd_rn(dot, __fmul_rn(x[i], w[i]));
  return dot;
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

// One warp per token.  bounds == nullptr means the logits are exact inputs
// (route-from-logits): no certification is needed.  When bounds is given,
// W and x must be the router weights and inputs the logits came from.
// stats[0] counts tokens that needed an exact recomputation.
template <int PL>
__global__ void __launch_bounds__(128)
    router_topk_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                       const float* __restrict__ bounds, int32_t* __restrict__ ids, float* __restrict__ probs, int H,
                       int E, int K, int T, int* __restrict__ stats) {
  const int lane = threadIdx.x & 31;
  const int wl = threadIdx.x >> 5;
  const int t = blockIdx.x * (blockDim.x >> 5) + wl;
  if (t >= T) return;
  __shared__ int s_cand[4][kMaxCandidates];
  __shared__ float s_val[4][kMaxCandidates];
  __shared__ int s_flag[4][kMaxCandidates];
  int* cand = s_cand[wl];
  float* cval = s_val[wl];
  int* flag = s_flag[wl];

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
    // Lowest lower bound among the chosen experts.
    float lowest_lo = INFINITY;
#pragma unroll
    for (int m = 0; m < PL; ++m)
      if (taken >> m & 1u) lowest_lo = fminf(lowest_lo, val[m] - bnd[m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lowest_lo = fminf(lowest_lo, __shfl_xor_sync(0xffffffffu, lowest_lo, o));

    // Candidate set Z = chosen experts plus every expert whose upper bound
    // reaches lowest_lo: every other expert is below all K chosen ones in the
    // reference too, so the reference's top-K lies in Z.
    count = K;
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
        }
      }
      count += __popc(mask);
    }
    __syncwarp();

    bool recomputed = false;
    if (count <= kMaxCandidates) {
      // Exact values for every candidate whose interval meets another's.
      for (int i = lane; i < count; i += 32) {
        const int ei = cand[i];
        const float ci = cval[i], bi_ = brow[ei];
        bool overlap = false;
        for (int j = 0; j < count; ++j) {
          if (j == i) continue;
          const float cj = cval[j], bj = brow[cand[j]];
          if (!(ci - bi_ > cj + bj || cj - bj > ci + bi_)) overlap = true;
        }
        flag[i] = overlap;
      }
      __syncwarp();
      for (int i = lane; i < count; i += 32) {
        if (flag[i]) {
          const int e = cand[i];
          const float v = exact_logit(x + (size_t)t * H, W + (size_t)e * H, H);
          cval[i] = v;
          lrow[e] = v;
          recomputed = true;
        }
      }
      __syncwarp();
      // Order Z by (value desc, id asc).  Every pair is either separated by
      // its bounds or compared on exact values: this is the reference order.
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
    } else {
      // Bounds too wide to certify anything: exact values for all experts.
      recomputed = true;
#pragma unroll
      for (int m = 0; m < PL; ++m) {
        const int e = lane + 32 * m;
        if (e < E) {
          val[m] = exact_logit(x + (size_t)t * H, W + (size_t)e * H, H);
          lrow[e] = val[m];
        }
      }
      warp_topk<PL>(val, E, K, cand, cval, taken);
    }
    recomputed = __any_sync(0xffffffffu, recomputed);
    if (recomputed && lane == 0 && stats) atomicAdd(stats, 1);
    __syncwarp();
  }

  // model.rs:1819-1829: p_k = expf(l_k - l_0), summed in k order, then
  // divided by max(sum, 1e-6).
  if (lane == 0) {
    const float max_l = cval[0];
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum = __fadd_rn(sum, exp_f32(__fsub_rn(cval[k], max_l)));
    const float denom = sum > 1e-6f ? sum : 1e-6f;
    for (int k = 0; k < K; ++k) {
      ids[(size_t)t * K + k] = cand[k];
      probs[(size_t)t * K + k] = __fdiv_rn(exp_f32(__fsub_rn(cval[k], max_l)), denom);
    }
  }
}


}  // namespace mrml

// ------------------------------------------------------------ launchers ---
namespace mrml {

cudaError_t launch_router_logits(const float* W, const float* x, float* logits, float* bounds, int H, int E, int T,
                                 cudaStream_t s) {
  const int tpc = T < 64 ? T : 64;
  const dim3 grid(E, (T + tpc - 1) / tpc);
  const size_t smem = (size_t)32 * ((H + 31) / 32 + 1) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t st = cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
  }
  router_logits_kernel<<<grid, 32 * kRouterWarps, smem, s>>>(W, x, logits, bounds, H, E, T, tpc);
  return cudaPeekAtLastError();
}

cudaError_t launch_router_topk(const float* W, const float* x, float* logits, const float* bounds, int32_t* ids,
                               float* probs, int H, int E, int K, int T, int* stats, cudaStream_t s) {
  const dim3 grid((T + 3) / 4);
  if (E <= 32)
    router_topk_kernel<1><<<grid, 128, 0, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, stats);
  else if (E <= 128)
    router_topk_kernel<4><<<grid, 128, 0, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, stats);
  else
    router_topk_kernel<8><<<grid, 128, 0, s>>>(W, x, logits, bounds, ids, probs, H, E, K, T, stats);
  return cudaPeekAtLastError();
}

}  // namespace mrml
