// topk.cuh — warp-level top-K and the reference's softmax tail, shared by
// the router's top-k kernel and the small-batch dispatch kernel.
#pragma once
#include "common.cuh"

namespace mrml {

constexpr int kMaxCandidates = 64;  // the largest supported K

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

// The reference's softmax over a token's K selected experts, already ordered
// by (value desc, id asc) in cand / cval (one warp):
// model.rs:1819-1829: p_k = expf(l_k - l_0), summed in k order, then divided
// by max(sum, 1e-6).  Lanes compute the exponentials in parallel; lane 0
// adds them in k order.
__device__ inline void softmax_sorted(const int* cand, float* cval, int K, int t, int32_t* ids, float* probs) {
  const int lane = threadIdx.x & 31;
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

// Per-token selection tail: order Z (count candidates) by (value desc, id
// asc), then the reference's softmax over the first K.
__device__ inline void finish_token(int* cand, float* cval, int count, int K, int t, int32_t* ids, float* probs) {
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
  softmax_sorted(cand, cval, K, t, ids, probs);
}

}  // namespace mrml
