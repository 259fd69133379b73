// experts.cu — token dispatch, grouped expert products and combine for the
// MRML MoE layer on sm_100a.
//
// Reference arithmetic (crates/mrml-tensor): the layer input of each token is
// quantised to Q8_0 (quant.rs:193-228, called at model.rs:2114-2115); every
// expert row is a block dot sum += (float)isum_b * (d_w * d_a) over the quant
// blocks in order (quant.rs:335-369, 564-577); act = geglu(gate, up)
// (ops.rs:99-114) is re-quantised to Q8_0 before the down rows (ops.rs:
// 175-177); the combine adds alpha*down*scale[e] slot by slot (model.rs:
// 2117-2165), skipping slots with alpha <= 1e-4.
//
// The f32 accumulation is kept in the reference's block order, without
// contraction, because act is re-quantised: any reordering of that sum flips
// int8 roundings of act and moves the layer output by up to ~5e-4 relative.
//
// B200 design: the reference re-streams an expert's weights once per
// (token, slot).  Here (token, slot) pairs are first grouped by expert
// (a stable counting sort), and each CTA streams one tile of one expert's
// rows from HBM exactly once with the TMA bulk-copy engine, then applies it
// to every token routed to that expert.  Integer block dots use dp4a; the
// int32 block sum becomes an f32 through the 1.5*2^23 bit trick.
#include <cfloat>
#include <initializer_list>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace mrml {

// ---------------------------------------------------------------------------
// Q8_0 quantisation of the layer input (quant.rs:193-228), one warp per
// 32-element block, lane = element.  Output in a GPU layout: int8 values
// [T][H], the decoded f16 scale d [T][H/32] as f32, and the block's sum of
// q values [T][H/32] (used to fold the Q4_0 "-8" offset into the dot).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quantize_block_warp(float v, int8_t* q_out, float* d_out, int32_t* sum_out,
                                                    uint32_t* d16_out) {
  const int lane = threadIdx.x & 31;
  float amax = fabsf(v);
  if (!(amax > 0.f)) amax = 0.f;  // `a > max_val` ignores NaN
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const uint32_t d16 = f32_to_f16_trunc(scale);
  const float id = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  float r = round_half_away(__fmul_rn(v, id));
  if (r != r) r = 0.f;
  r = fminf(fmaxf(r, -128.f), 127.f);
  const int q = (int)r;
  q_out[lane] = (int8_t)q;
  int s = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    if (d_out) *d_out = f16_bits_to_f32(d16);
    if (sum_out) *sum_out = s;
    if (d16_out) *d16_out = d16;
  }
}

__global__ void quantize_rows_kernel(const float* __restrict__ x, int8_t* __restrict__ xq, float* __restrict__ xd,
                                     int32_t* __restrict__ xsum, long long n_blocks) {
  pdl_trigger();
  pdl_wait();
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
    const float v = x[b * 32 + (threadIdx.x & 31)];
    quantize_block_warp(v, xq + b * 32, xd + b, xsum + b, nullptr);
  }
}

// GGUF-format quantisers (block bytes exactly as the reference writes them).
__global__ void quantize_q8_0_gguf_kernel(const float* __restrict__ x, uint8_t* __restrict__ dst, long long n_blocks) {
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
    __shared__ int8_t q[8][32];
    const int w = threadIdx.x >> 5;
    uint32_t d16 = 0;
    quantize_block_warp(x[b * 32 + lane], q[w], nullptr, nullptr, &d16);
    d16 = __shfl_sync(0xffffffffu, d16, 0);
    __syncwarp();
    uint8_t* o = dst + b * 34;
    if (lane < 2) o[lane] = (uint8_t)(lane == 0 ? d16 & 0xff : d16 >> 8);
    o[2 + lane] = (uint8_t)q[w][lane];
    __syncwarp();
  }
}

// quant.rs:372-389: d = max|v| / 8 (truncating f16), q = clamp(round(v/d),
// -8, 7) + 8, low nibble = element j, high nibble = element j + 16.
__global__ void quantize_q4_0_gguf_kernel(const float* __restrict__ x, uint8_t* __restrict__ dst, long long n_blocks) {
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
    const float v = x[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.f ? __fdiv_rn(amax, 8.0f) : 0.f;
    const uint32_t d16 = f32_to_f16_trunc(scale);
    const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
    float r = round_half_away(__fmul_rn(v, inv));
    if (r != r) r = 0.f;
    const int q = (int)fminf(fmaxf(r, -8.f), 7.f) + 8;
    const int hi = __shfl_down_sync(0xffffffffu, q, 16);
    uint8_t* o = dst + b * 18;
    if (lane < 16) o[2 + lane] = (uint8_t)(q | (hi << 4));
    if (lane < 2) o[lane] = (uint8_t)(lane == 0 ? d16 & 0xff : d16 >> 8);
  }
}

// Token t's block b quantised to Q8_0 (quant.rs:193-228) and stored at every
// position the token was routed to (quantize_scatter_kernel's layout); one
// warp, lane = element.
template <int WQ4>
__device__ __forceinline__ void quantize_scatter_block(const float* __restrict__ x, const int32_t* __restrict__ pos,
                                                       int t, int b, int H, int K, int npad, int group_major,
                                                       int8_t* __restrict__ bq, int2* __restrict__ bsc) {
  const int nb = H / 32, lane = threadIdx.x & 31;
  const float v = x[(size_t)t * H + b * 32 + lane];
  float amax = fabsf(v);
  if (!(amax > 0.f)) amax = 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const uint32_t d16 = f32_to_f16_trunc(scale);
  const float id = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  float r = round_half_away(__fmul_rn(v, id));
  if (r != r) r = 0.f;
  r = fminf(fmaxf(r, -128.f), 127.f);
  const int q = (int)r;
  int qsum = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
  const int2 sc = make_int2(__float_as_int(f16_bits_to_f32(d16)), WQ4 ? kMagicI - 8 * qsum : kMagicI);
  for (int k = 0; k < K; ++k) {
    const int p = pos[t * K + k];
    if (p < 0) continue;
    uint8_t* dst = reinterpret_cast<uint8_t*>(bq) + act_group_offset(group_major, b, p >> 3, nb, npad) +
                   (lane >> 4) * 128 + (p & 7) * 16 + (lane & 15);
    *dst = (uint8_t)(int8_t)q;
    if (lane == 0) {
      if (group_major)
        store_act_scale_gm(bsc, b, p, nb, __int_as_float(sc.x), sc.y);
      else
        bsc[act_scale_index(b, p, npad)] = sc;
    }
  }
}

// ---------------------------------------------------------------------------
// Dispatch: a stable counting sort of the (token, slot) pairs p = t*K + k by
// expert id, skipping slots with alpha <= 1e-4 (model.rs:2119).  Each
// expert's segment of the sorted order is padded to a multiple of 16
// positions (tensor-core token tiles start on 8-position core-matrix
// boundaries).  Produces cnt[E], poff[E+1] (padded segment starts),
// pair_at[poff[E]] (the pair at each position, -1 for padding) and
// pos[T*K] (each pair's position, -1 if skipped), and the work-unit tables
// of the tensor-core products: units_gu / units_dn hold {e, first position,
// valid positions, first weight row} per (expert, 128-row tile, NT-position
// tile; gate/up tiles have rows_gu rows, down tiles 128); n_units =
// {#gate/up units, #down units}.
// One CTA of 1024 threads; pairs are ranked chunk by chunk with warp match.
// ---------------------------------------------------------------------------
constexpr int kDispatchThreads = 1024;

// ---------------------------------------------------------------------------
// Speculative selection of one token's experts (one warp; E <= 256).  With
// intervals [lo_e, hi_e] that contain the reference's router logits, the
// experts whose hi_e reaches tau, the K-th largest lo, contain the reference's
// top-K: an expert e with hi_e < tau lies strictly below K others.  They
// become the token's candidate slots ids[t*C + j] (expert ids ascending,
// weight 1; unused slots weight 0, which the counting sort skips).  When more
// than C experts qualify (logits within the rounding bound of one another, or
// a bound that is not finite), the warp computes the token's exact logits with
// the router kernel's chain and takes the exact top-K (warp_topk, the router's
// own selection).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exact_router_logit(const float* __restrict__ w, const float* __restrict__ x, int H) {
  float acc = 0.f;
  for (int i = 0; i < H; ++i) acc = __fadd_rn(acc, __fmul_rn(x[i], w[i]));
  return acc;
}

__device__ void spec_select_token(const SpecRoute& S, int E, int t, int* cand, float* cval, int32_t* ids,
                                  float* probs) {
  const unsigned int full = 0xffffffffu;
  const int lane = threadIdx.x & 31, C = S.C, K = S.K;
  float lo[8], hi[8];
  bool bad = false;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int e = lane + 32 * m;
    lo[m] = e < E ? S.lo[(size_t)t * E + e] : -INFINITY;
    hi[m] = e < E ? S.hi[(size_t)t * E + e] : -INFINITY;
    if (e < E && !(fabsf(lo[m]) <= FLT_MAX && fabsf(hi[m]) <= FLT_MAX)) bad = true;
  }
  bad = __any_sync(full, bad);
  uint32_t taken;
  int count = 0;
  float tau = 0.f;
  if (!bad) {
    warp_topk<8>(lo, E, K, cand, cval, taken);
    tau = cval[K - 1];
#pragma unroll
    for (int m = 0; m < 8; ++m) count += __popc(__ballot_sync(full, lane + 32 * m < E && hi[m] >= tau));
  }
  __syncwarp();
  if (!bad && count <= C) {
    int j = 0;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int e = lane + 32 * m;
      const bool in = e < E && hi[m] >= tau;
      const unsigned int b = __ballot_sync(full, in);
      if (in) {
        const int slot = j + __popc(b & ((1u << lane) - 1u));
        ids[(size_t)t * C + slot] = e;
        probs[(size_t)t * C + slot] = 1.0f;
      }
      j += __popc(b);
    }
    for (int slot = count + lane; slot < C; slot += 32) {
      ids[(size_t)t * C + slot] = 0;
      probs[(size_t)t * C + slot] = 0.f;
    }
    return;
  }
  float val[8];
#pragma unroll 1
  for (int m = 0; m < 8; ++m) {
    const int e = lane + 32 * m;
    val[m] = e < E ? exact_router_logit(S.W + (size_t)e * S.H, S.x + (size_t)t * S.H, S.H) : -INFINITY;
  }
  warp_topk<8>(val, E, K, cand, cval, taken);
  for (int slot = lane; slot < C; slot += 32) {
    ids[(size_t)t * C + slot] = slot < K ? cand[slot] : 0;
    probs[(size_t)t * C + slot] = slot < K ? 1.0f : 0.f;
  }
}


//
// With `logits` (small batches: T = n_pairs / K <= kDispatchTopkMaxTokens, E <= 256) the
// kernel first selects each token's experts itself and writes ids and probs;
// the rest of the kernel reads them back (global writes of the CTA are
// visible to it after the barrier).  That saves the top-k launch on the
// decode path.  The selection is router_topk_kernel's (one warp per token,
// warp top-k, then the reference's softmax), or for the smallest batches the
// same ordering computed by rank.
__global__ void __launch_bounds__(kDispatchThreads)
    dispatch_kernel(int32_t* ids, float* probs, int n_pairs, int E, int e_first, int e_total,
                    int32_t* __restrict__ cnt_out, int32_t* __restrict__ poff, int32_t* __restrict__ pair_at,
                    int32_t* __restrict__ pos, int4* __restrict__ units_gu, int4* __restrict__ units_dn,
                    int* __restrict__ n_units, int NT_gu, int NT_dn, int mt_gu, int rows_gu, int mt_dn,
                    int* __restrict__ err, const float* __restrict__ logits, int K, SpecRoute spec) {
  pdl_trigger();
  // Dynamic shared memory: the counting sort's arrays, then, when the kernel
  // selects the experts, each warp's slots.
  extern __shared__ int32_t dsm[];
  const int WS = E + 1;          // row stride of wcnt (odd: the scan's column reads hit distinct banks)
  int32_t* cnt = dsm;            // [E] totals
  int32_t* base = dsm + E;       // [E] running position of the next pair of expert e
  int32_t* ubase = dsm + 2 * E;  // [E] first gate/up unit of expert e (times mt)
  int32_t* ubase_dn = dsm + 3 * E;  // [E] first down unit of expert e (times mt)
  int32_t* wcnt = dsm + 4 * E;   // [32][WS] per-warp counts of the current chunk
  __shared__ int s_npos;         // positions in use (padded segments)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Shared memory is this CTA's own: cleared while the previous kernel ends.
  for (int i = tid; i < 4 * E + 32 * WS; i += blockDim.x) dsm[i] = 0;
  pdl_wait();
  if (spec.lo != nullptr) {
    const int T = n_pairs / spec.C;
    int* tk_cand = dsm + 4 * E + 32 * WS;                          // [32][K] one warp's slots
    float* tk_cval = reinterpret_cast<float*>(tk_cand + 32 * spec.K);  // [32][K]
    for (int t = warp; t < T; t += kDispatchThreads / 32)
      spec_select_token(spec, E, t, tk_cand + warp * spec.K, tk_cval + warp * spec.K, ids, probs);
  } else if (logits != nullptr && (n_pairs / K) * E <= kDispatchRankSelectMax) {
    // The smallest batches select by rank: with the logits in shared memory,
    // the thread of (t, e) counts the experts that come before e in the
    // (value desc, id asc) order, and an expert of rank r < K lands in slot
    // r; one warp per token then runs the reference's softmax over the slots.
    // (Measured on B200 at config 2: 12.9 against 15.5 us for the warp top-k
    // at T = 1; at T = 8 the warp top-k is ahead.)
    const int T = n_pairs / K;
    float* lg = reinterpret_cast<float*>(dsm + 4 * E + 32 * WS);  // [T][E]
    int* tk_cand = reinterpret_cast<int*>(lg + T * E);             // [T][K] experts by rank
    float* tk_cval = reinterpret_cast<float*>(tk_cand + T * K);    // [T][K] their logits
    for (int i = tid; i < T * E; i += blockDim.x) lg[i] = logits[i];
    __syncthreads();
    for (int i = tid; i < T * E; i += blockDim.x) {
      const int t = i / E, e = i - t * E;
      const float v = lg[i];
      const float* row = lg + t * E;
      int r = 0;
      for (int f = 0; f < E; ++f) {
        const float u = row[f];
        r += (u > v || (u == v && f < e)) ? 1 : 0;
      }
      if (r < K) {
        tk_cand[t * K + r] = e;
        tk_cval[t * K + r] = v;
      }
    }
    __syncthreads();
    if (warp < T) softmax_sorted(tk_cand + warp * K, tk_cval + warp * K, K, warp, ids, probs);
  } else if (logits != nullptr) {
    const int T = n_pairs / K;
    int* tk_cand = dsm + 4 * E + 32 * WS;                          // [32][K] one warp's slots
    float* tk_cval = reinterpret_cast<float*>(tk_cand + 32 * K);   // [32][K]
    for (int t = warp; t < T; t += kDispatchThreads / 32) {
      float val[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int e = lane + 32 * m;
        val[m] = e < E ? logits[(size_t)t * E + e] : -INFINITY;
      }
      uint32_t taken;
      warp_topk<8>(val, E, K, tk_cand + warp * K, tk_cval + warp * K, taken);
      finish_token(tk_cand + warp * K, tk_cval + warp * K, K, K, t, ids, probs);
    }
  }
  __syncthreads();
  // The thread's first pair, read once for the count and the scatter.
  int id0 = 0;
  float p0 = 0.f;
  if (tid < n_pairs) {
    id0 = ids[tid];
    p0 = probs[tid];
  }
  // Experts [e_first, e_first + E) of e_total are this call's; pairs routed
  // to the others are skipped like pairs with alpha <= 1e-4 (an expert-
  // parallel shard), ids outside [0, e_total) are errors.
  for (int p = tid; p < n_pairs; p += blockDim.x) {
    const int id = p == tid ? id0 : ids[p];
    if ((p == tid ? p0 : probs[p]) > 0.0001f) {
      if (id < 0 || id >= e_total)
        set_error(err, kDevBadExpert);
      else if (id - e_first >= 0 && id - e_first < E)
        atomicAdd(&cnt[id - e_first], 1);
    }
  }
  __syncthreads();
  // Exclusive scans of the padded counts and of the two products' unit
  // counts, one warp per 32 experts, then across warps (E <= 1024).
  {
    __shared__ int wsum_pos[32], wsum_units[32], wsum_dn[32];
    const int e = tid;
    const int c = e < E ? cnt[e] : 0;
    const int pad = (c + 15) & ~15, nun = (c + NT_gu - 1) / NT_gu, nud = (c + NT_dn - 1) / NT_dn;
    int ip = pad, iu = nun, id = nud;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vp = __shfl_up_sync(0xffffffffu, ip, o), vu = __shfl_up_sync(0xffffffffu, iu, o);
      const int vd = __shfl_up_sync(0xffffffffu, id, o);
      if (lane >= o) {
        ip += vp;
        iu += vu;
        id += vd;
      }
    }
    if (lane == 31) {
      wsum_pos[warp] = ip;
      wsum_units[warp] = iu;
      wsum_dn[warp] = id;
    }
    __syncthreads();
    if (warp == 0) {
      int vp = wsum_pos[lane], vu = wsum_units[lane], vd = wsum_dn[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, vp, o), b = __shfl_up_sync(0xffffffffu, vu, o);
        const int d = __shfl_up_sync(0xffffffffu, vd, o);
        if (lane >= o) {
          vp += a;
          vu += b;
          vd += d;
        }
      }
      wsum_pos[lane] = vp;  // inclusive per warp
      wsum_units[lane] = vu;
      wsum_dn[lane] = vd;
    }
    __syncthreads();
    const int bp = warp ? wsum_pos[warp - 1] : 0, bu = warp ? wsum_units[warp - 1] : 0;
    const int bd = warp ? wsum_dn[warp - 1] : 0;
    if (e < E) {
      poff[e] = bp + ip - pad;
      base[e] = bp + ip - pad;
      ubase[e] = bu + iu - nun;
      ubase_dn[e] = bd + id - nud;
      cnt_out[e] = c;
    }
    if (e == E - 1) {
      poff[E] = bp + ip;
      s_npos = bp + ip;
      n_units[0] = (bu + iu) * mt_gu;
      n_units[1] = (bd + id) * mt_dn;
    }
  }
  __syncthreads();
  const int npos = s_npos;
  for (int i = tid; i < npos; i += blockDim.x) pair_at[i] = -1;
  // Work units: expert e owns units [ubase[e]*mt, (ubase[e] + nt_e)*mt) of
  // each product, ordered (row tile m, position tile j), j fastest.
  // kDispatchThreads / E threads per expert write its units.  base[] still
  // holds the segment starts here.
  {
    const int per = kDispatchThreads / E, e = tid / per, sub = tid - e * per;
    if (e < E) {
      const int c = cnt[e];
      for (int prod = 0; prod < 2; ++prod) {
        const int mt = prod == 0 ? mt_gu : mt_dn, rows = prod == 0 ? rows_gu : 128;
        const int NT = prod == 0 ? NT_gu : NT_dn;
        const int first = (prod == 0 ? ubase : ubase_dn)[e] * mt, nt = (c + NT - 1) / NT;
        int4* units = prod == 0 ? units_gu : units_dn;
        for (int local = sub; local < nt * mt; local += per) {
          const int m = local / nt, j = local - m * nt;
          units[first + local] = make_int4(e, base[e] + j * NT, min(NT, c - j * NT), m * rows);
        }
      }
    }
  }
  __syncthreads();
  // Stable scatter, 1024 pairs at a time.
  for (int b0 = 0; b0 < n_pairs; b0 += blockDim.x) {
    const int p = b0 + tid;
    int e = -1;
    if (p < n_pairs) {
      const int id = (b0 == 0 ? id0 : ids[p]) - e_first;
      if ((b0 == 0 ? p0 : probs[p]) > 0.0001f && id >= 0 && id < E && id + e_first < e_total) e = id;
      if (e < 0) pos[p] = -1;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp * WS + e] = __popc(peers);
    __syncthreads();
    // per expert, an exclusive scan over the 32 warps' counts (lane = warp)
    for (int x = warp; x < E; x += 32) {
      const int c = wcnt[lane * WS + x];
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int b = base[x];
      wcnt[lane * WS + x] = b + incl - c;
      __syncwarp();
      if (lane == 31) base[x] = b + incl;
    }
    __syncthreads();
    if (e >= 0) {
      const int dst = wcnt[warp * WS + e] + rank;
      pair_at[dst] = p;
      pos[p] = dst;
    }
    __syncthreads();
    for (int i = tid; i < 32 * WS; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Dispatch for the smallest batches (at most 32 pairs): the same outputs as
// dispatch_kernel (stable counting sort by expert, segments padded to 16,
// work units, the selection when asked), computed
// without the block-wide scans: warp 0 holds one pair per lane, finds each
// expert's pairs with a warp match and each segment's start by summing the
// padded counts of the experts before it over the lanes; the other warps
// then write the per-expert tables and the work units.
// ---------------------------------------------------------------------------
constexpr int kDispatchSmallThreads = 512;
constexpr int kDispatchSmallPairs = 32;

__global__ void __launch_bounds__(kDispatchSmallThreads)
    dispatch_small_kernel(int32_t* ids, float* probs, int n_pairs, int E, int e_first, int e_total,
                          int32_t* __restrict__ cnt_out, int32_t* __restrict__ poff, int32_t* __restrict__ pair_at,
                          int32_t* __restrict__ pos, int4* __restrict__ units_gu, int4* __restrict__ units_dn,
                          int* __restrict__ n_units, int NT_gu, int NT_dn, int mt_gu, int rows_gu, int mt_dn,
                          int* __restrict__ err, const float* __restrict__ logits, int K, SpecRoute spec) {
  extern __shared__ float lg[];  // [T][E] logits (selection)
  __shared__ int s_cand[kDispatchSmallPairs];
  __shared__ float s_cval[kDispatchSmallPairs];
  __shared__ int s_e[kDispatchSmallPairs], s_c[kDispatchSmallPairs], s_base[kDispatchSmallPairs];
  __shared__ int s_ugu[kDispatchSmallPairs], s_udn[kDispatchSmallPairs], s_pos[kDispatchSmallPairs];
  __shared__ int s_nlead, s_npos;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  pdl_trigger();
  pdl_wait();
  if (spec.lo != nullptr) {
    // T * C <= 32: each token's K slots fit in s_cand / s_cval
    if (warp < n_pairs / spec.C)
      spec_select_token(spec, E, warp, s_cand + warp * spec.K, s_cval + warp * spec.K, ids, probs);
    __syncthreads();
  } else if (logits != nullptr) {
    const int T = n_pairs / K;
    for (int i = tid; i < T * E; i += blockDim.x) lg[i] = logits[i];
    __syncthreads();
    // rank of (t, e) in the (value desc, id asc) order (router_topk_kernel's)
    for (int i = tid; i < T * E; i += blockDim.x) {
      const int t = i / E, e = i - t * E;
      const float v = lg[i];
      const float* row = lg + t * E;
      int r = 0;
      for (int f = 0; f < E; ++f) {
        const float u = row[f];
        r += (u > v || (u == v && f < e)) ? 1 : 0;
      }
      if (r < K) {
        s_cand[t * K + r] = e;
        s_cval[t * K + r] = v;
      }
    }
    __syncthreads();
    if (warp < T) softmax_sorted(s_cand + warp * K, s_cval + warp * K, K, warp, ids, probs);
    __syncthreads();
  }
  if (warp == 0) {
    const unsigned int full = 0xffffffffu;
    const bool have = lane < n_pairs;
    const int id = have ? ids[lane] : 0;
    const float pr = have ? probs[lane] : 0.f;
    int e = -1;
    if (have && pr > 0.0001f) {
      if (id < 0 || id >= e_total)
        set_error(err, kDevBadExpert);
      else if (id - e_first >= 0 && id - e_first < E)
        e = id - e_first;
    }
    const unsigned int grp = __match_any_sync(full, e);
    const int c = __popc(grp), rk = __popc(grp & ((1u << lane) - 1u));
    const bool lead = e >= 0 && rk == 0;
    int base = 0, ugu = 0, udn = 0, npos = 0, tgu = 0, tdn = 0;
    for (int q = 0; q < 32; ++q) {
      const int eq = __shfl_sync(full, e, q), cq = __shfl_sync(full, c, q);
      if (__shfl_sync(full, lead ? 1 : 0, q)) {
        const int pad = (cq + 15) & ~15, nug = (cq + NT_gu - 1) / NT_gu, nud = (cq + NT_dn - 1) / NT_dn;
        if (eq < e) {
          base += pad;
          ugu += nug;
          udn += nud;
        }
        npos += pad;
        tgu += nug;
        tdn += nud;
      }
    }
    const int p_here = e >= 0 ? base + rk : -1;
    if (have) pos[lane] = p_here;
    s_pos[lane] = p_here;
    const unsigned int lm = __ballot_sync(full, lead);
    if (lead) {
      const int slot = __popc(lm & ((1u << lane) - 1u));
      s_e[slot] = e;
      s_c[slot] = c;
      s_base[slot] = base;
      s_ugu[slot] = ugu;
      s_udn[slot] = udn;
    }
    if (lane == 0) {
      s_nlead = __popc(lm);
      s_npos = npos;
      n_units[0] = tgu * mt_gu;
      n_units[1] = tdn * mt_dn;
    }
  }
  __syncthreads();
  const int nl = s_nlead, npos = s_npos;
  for (int x = tid; x <= E; x += blockDim.x) {
    int cx = 0, px = 0;
    for (int j = 0; j < nl; ++j) {
      if (s_e[j] == x) cx = s_c[j];
      if (s_e[j] < x) px += (s_c[j] + 15) & ~15;
    }
    if (x < E) cnt_out[x] = cx;
    poff[x] = px;
  }
  for (int i = tid; i < npos; i += blockDim.x) pair_at[i] = -1;
  __syncthreads();
  if (tid < n_pairs && s_pos[tid] >= 0) pair_at[s_pos[tid]] = tid;
  // work units of each present expert: (row tile m, position tile j), j fastest
  for (int j = warp; j < nl; j += nwarps) {
    const int e = s_e[j], c = s_c[j], b = s_base[j];
    for (int prod = 0; prod < 2; ++prod) {
      const int mt = prod == 0 ? mt_gu : mt_dn, rows = prod == 0 ? rows_gu : 128;
      const int NT = prod == 0 ? NT_gu : NT_dn, ub = prod == 0 ? s_ugu[j] : s_udn[j];
      const int nt = (c + NT - 1) / NT;
      int4* units = prod == 0 ? units_gu : units_dn;
      for (int local = lane; local < nt * mt; local += 32) {
        const int m = local / nt, jj = local - m * nt;
        units[ub * mt + local] = make_int4(e, b + jj * NT, min(NT, c - jj * NT), m * rows);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Dispatch for large batches, in three launches over chunks of
// kDispatchThreads pairs (the single-CTA kernel above walks the chunks one
// after another; at 65k pairs that alone took ~0.3 ms).  The result is the
// same stable counting sort, bit for bit: positions ordered by expert, then
// by pair index.
//   count:   one CTA per chunk counts its pairs per expert -> chunk_cnt[c][E];
//   layout:  one CTA turns the counts into each chunk's first position per
//            expert (in place), the totals, the padded segment starts, the
//            work-unit tables and the padding markers (the single-CTA
//            kernel's scans, over experts);
//   scatter: one CTA per chunk ranks its pairs per expert in pair order
//            (warp match, then per-warp counts scanned across the CTA's warps)
//            and writes pair_at / pos.
// ---------------------------------------------------------------------------

// Pair p's local expert (id - e_first) when it is one of this call's pairs
// (alpha > 1e-4 and an id in the call's experts), else -1; ids outside
// [0, e_total) are reported.
__device__ __forceinline__ int pair_expert(const int32_t* ids, const float* probs, int p, int E, int e_first,
                                           int e_total, int* err, bool report) {
  if (!(probs[p] > 0.0001f)) return -1;
  const int id = ids[p];
  if (id < 0 || id >= e_total) {
    if (report) set_error(err, kDevBadExpert);
    return -1;
  }
  const int e = id - e_first;
  return e >= 0 && e < E ? e : -1;
}

__global__ void __launch_bounds__(kDispatchThreads)
    dispatch_count_kernel(const int32_t* __restrict__ ids, const float* __restrict__ probs, int n_pairs, int E,
                          int e_first, int e_total, int32_t* __restrict__ chunk_cnt, int* __restrict__ err) {
  extern __shared__ int32_t ccnt[];  // [E]
  for (int i = threadIdx.x; i < E; i += blockDim.x) ccnt[i] = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int p = blockIdx.x * kDispatchThreads + threadIdx.x;
  if (p < n_pairs) {
    const int e = pair_expert(ids, probs, p, E, e_first, e_total, err, true);
    if (e >= 0) atomicAdd(&ccnt[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) chunk_cnt[(size_t)blockIdx.x * E + i] = ccnt[i];
}

constexpr int kLayoutTile = 32;  // chunks per shared-memory tile of the layout step

__global__ void __launch_bounds__(kDispatchThreads)
    dispatch_layout_kernel(int32_t* __restrict__ chunk_cnt, int nchunks, int E, int32_t* __restrict__ cnt_out,
                           int32_t* __restrict__ poff, int32_t* __restrict__ pair_at, int4* __restrict__ units_gu,
                           int4* __restrict__ units_dn, int* __restrict__ n_units, int NT_gu, int NT_dn, int mt_gu,
                           int rows_gu, int mt_dn) {
  extern __shared__ int32_t lsm[];
  int32_t* cnt = lsm;                // [E]
  int32_t* base = lsm + E;           // [E] segment start
  int32_t* ubase = lsm + 2 * E;      // [E] first gate/up unit (times mt)
  int32_t* ubase_dn = lsm + 3 * E;   // [E] first down unit (times mt)
  int32_t* tile = lsm + 4 * E;       // [kLayoutTile][E] chunk counts being scanned
  __shared__ int s_npos;
  __shared__ int wsum_pos[32], wsum_units[32], wsum_dn[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  // Per expert: each chunk's offset within the expert's pairs (exclusive
  // prefix over chunks, written back in place) and the expert's total.  The
  // counts move through shared memory kLayoutTile chunks at a time with
  // coalesced loads and stores, so that no thread walks global memory in a
  // dependent chain.
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  for (int c0 = 0; c0 < nchunks; c0 += kLayoutTile) {
    const int nc = min(kLayoutTile, nchunks - c0);
    __syncthreads();
    for (int i = tid; i < nc * E; i += blockDim.x) tile[i] = chunk_cnt[(size_t)c0 * E + i];
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
      int run = cnt[e];
      for (int c = 0; c < nc; ++c) {
        const int v = tile[c * E + e];
        tile[c * E + e] = run;
        run += v;
      }
      cnt[e] = run;
    }
    __syncthreads();
    for (int i = tid; i < nc * E; i += blockDim.x) chunk_cnt[(size_t)c0 * E + i] = tile[i];
  }
  __syncthreads();
  {
    const int e = tid;
    const int c = e < E ? cnt[e] : 0;
    const int pad = (c + 15) & ~15, nun = (c + NT_gu - 1) / NT_gu, nud = (c + NT_dn - 1) / NT_dn;
    int ip = pad, iu = nun, id = nud;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vp = __shfl_up_sync(0xffffffffu, ip, o), vu = __shfl_up_sync(0xffffffffu, iu, o);
      const int vd = __shfl_up_sync(0xffffffffu, id, o);
      if (lane >= o) {
        ip += vp;
        iu += vu;
        id += vd;
      }
    }
    if (lane == 31) {
      wsum_pos[warp] = ip;
      wsum_units[warp] = iu;
      wsum_dn[warp] = id;
    }
    __syncthreads();
    if (warp == 0) {
      int vp = wsum_pos[lane], vu = wsum_units[lane], vd = wsum_dn[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, vp, o), b = __shfl_up_sync(0xffffffffu, vu, o);
        const int d = __shfl_up_sync(0xffffffffu, vd, o);
        if (lane >= o) {
          vp += a;
          vu += b;
          vd += d;
        }
      }
      wsum_pos[lane] = vp;
      wsum_units[lane] = vu;
      wsum_dn[lane] = vd;
    }
    __syncthreads();
    const int bp = warp ? wsum_pos[warp - 1] : 0, bu = warp ? wsum_units[warp - 1] : 0;
    const int bd = warp ? wsum_dn[warp - 1] : 0;
    if (e < E) {
      poff[e] = bp + ip - pad;
      base[e] = bp + ip - pad;
      ubase[e] = bu + iu - nun;
      ubase_dn[e] = bd + id - nud;
      cnt_out[e] = c;
    }
    if (e == E - 1) {
      poff[E] = bp + ip;
      s_npos = bp + ip;
      n_units[0] = (bu + iu) * mt_gu;
      n_units[1] = (bd + id) * mt_dn;
    }
  }
  __syncthreads();
  const int npos = s_npos;
  for (int i = tid; i < npos; i += blockDim.x) pair_at[i] = -1;
  for (int prod = 0; prod < 2; ++prod) {
    const int mt = prod == 0 ? mt_gu : mt_dn, rows = prod == 0 ? rows_gu : 128;
    const int NT = prod == 0 ? NT_gu : NT_dn;
    const int32_t* ub = prod == 0 ? ubase : ubase_dn;
    const int nu = ub[E - 1] + (cnt[E - 1] + NT - 1) / NT;
    int4* units = prod == 0 ? units_gu : units_dn;
    for (int u = tid; u < nu * mt; u += blockDim.x) {
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ub[mid] * mt <= u)
          lo = mid;
        else
          hi = mid - 1;
      }
      const int e = lo, c = cnt[e], nt = (c + NT - 1) / NT;
      const int local = u - ub[e] * mt, m = local / nt, j = local - m * nt;
      units[u] = make_int4(e, base[e] + j * NT, min(NT, c - j * NT), m * rows);
    }
  }
}

__global__ void __launch_bounds__(kDispatchThreads)
    dispatch_scatter_kernel(const int32_t* __restrict__ ids, const float* __restrict__ probs, int n_pairs, int E,
                            int e_first, int e_total, const int32_t* __restrict__ chunk_base,
                            const int32_t* __restrict__ poff, int32_t* __restrict__ pair_at,
                            int32_t* __restrict__ pos) {
  extern __shared__ int32_t wcnt[];  // [32][E] per-warp counts, then their exclusive prefix
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E; i += blockDim.x) wcnt[i] = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int p = blockIdx.x * kDispatchThreads + tid;
  int e = -1;
  if (p < n_pairs) {
    e = pair_expert(ids, probs, p, E, e_first, e_total, nullptr, false);
    if (e < 0) pos[p] = -1;
  }
  const uint32_t peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = tid; x < E; x += blockDim.x) {
    int run = poff[x] + chunk_base[(size_t)blockIdx.x * E + x];
    for (int w = 0; w < 32; ++w) {
      const int c = wcnt[w * E + x];
      wcnt[w * E + x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (e >= 0) {
    const int dst = wcnt[warp * E + e] + rank;
    pair_at[dst] = p;
    pos[p] = dst;
  }
}

// Q8_0 quantisation of the layer input scattered straight into the tensor-
// core B operand: for every position a token was routed to, its 32 int8
// values of block b go to bq[b][pos/8] in the canonical K-major layout (two
// 16-byte halves, core matrices of 8 positions), and {d, correction} to
// bsc[b][pos] (block-major), or into the group-major scale records of the
// decode kernel.  One warp per (token, block), lane = element.
template <int WQ4>
__global__ void quantize_scatter_kernel(const float* __restrict__ x, const int32_t* __restrict__ pos, int T, int H,
                                        int K, int npad, int group_major, int8_t* __restrict__ bq,
                                        int2* __restrict__ bsc) {
  // Waiting before triggering means that when the expert kernel that
  // follows starts, the dispatch kernel before this one has completed, so
  // that kernel may read its work units and stream weights right away.
  pdl_wait();
  pdl_trigger();
  const int nb = H / 32;
  const long long total = (long long)T * nb;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps)
    quantize_scatter_block<WQ4>(x, pos, (int)(w / nb), (int)(w % nb), H, K, npad, group_major, bq, bsc);
}

// Large batches: the layer input is quantised once per token
// (quantize_rows_kernel, the same quantiser), then this kernel builds the
// decode kernel's group-major operand one (position group, block) per warp:
// lane (j = lane / 4, part = lane % 4) copies 8 bytes of position j's row
// from its token, so the warp writes the group's whole 256-byte block and
// 96-byte scale record at once (the per-token scatter writes 16-byte
// pieces of blocks that other tokens complete later).  Padding positions
// get zero values and a zero scale.  Positions in use: poff[E].
__global__ void gather_groups_kernel(const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                     const int32_t* __restrict__ xsum, const int32_t* __restrict__ pair_at,
                                     const int32_t* __restrict__ poff_end, int H, int K, int wq4, int npad,
                                     int8_t* __restrict__ bq, int2* __restrict__ bsc) {
  // As quantize_scatter_kernel: wait, then trigger, so the expert kernel
  // that follows may read the dispatch kernel's work units right away.
  pdl_wait();
  pdl_trigger();
  const int nb = H / 32;
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
    uint8_t* dst = reinterpret_cast<uint8_t*>(bq) + act_group_offset(true, b, g, nb, npad) + (part >> 1) * 128 +
                   j * 16 + 8 * (part & 1);
    *reinterpret_cast<uint2*>(dst) = v;
    if (part == 0) {
      float d = 0.f;
      int corr = kMagicI;
      if (t >= 0) {
        d = xd[(size_t)t * nb + b];
        if (wq4) corr = kMagicI - 8 * xsum[(size_t)t * nb + b];
      }
      store_act_scale_gm(bsc, b, pos, nb, d, corr);
    }
  }
}

// ---------------------------------------------------------------------------
// One row-block product for `ntok` tokens is not done here; each thread runs
// one (row, token) chain over the row's blocks in order, as the reference
// does, so its f32 result is bit-identical to vec_dot_*.
// ---------------------------------------------------------------------------
template <int WT>
__device__ __forceinline__ float row_dot_chain(const uint8_t* __restrict__ row, int nb, const int8_t* __restrict__ aq,
                                               const float* __restrict__ ad, const int32_t* __restrict__ abias) {
  float sum = 0.f;
  for (int b = 0; b < nb; ++b) {
    const int4* av = reinterpret_cast<const int4*>(aq + b * 32);
    const int4 a0 = av[0], a1 = av[1];
    int acc = abias[b];
    uint32_t d16;
    if constexpr (WT == kQ4_0) {
      const Q4Block w = load_q4_block(row + b * 18);
      d16 = w.d16;
      acc = dp4a_us(w.qs[0] & 0x0f0f0f0fu, (uint32_t)a0.x, acc);
      acc = dp4a_us(w.qs[1] & 0x0f0f0f0fu, (uint32_t)a0.y, acc);
      acc = dp4a_us(w.qs[2] & 0x0f0f0f0fu, (uint32_t)a0.z, acc);
      acc = dp4a_us(w.qs[3] & 0x0f0f0f0fu, (uint32_t)a0.w, acc);
      acc = dp4a_us((w.qs[0] >> 4) & 0x0f0f0f0fu, (uint32_t)a1.x, acc);
      acc = dp4a_us((w.qs[1] >> 4) & 0x0f0f0f0fu, (uint32_t)a1.y, acc);
      acc = dp4a_us((w.qs[2] >> 4) & 0x0f0f0f0fu, (uint32_t)a1.z, acc);
      acc = dp4a_us((w.qs[3] >> 4) & 0x0f0f0f0fu, (uint32_t)a1.w, acc);
    } else {
      const Q8Block w = load_q8_block(row + b * 34);
      d16 = w.d16;
      acc = dp4a_ss(w.qs[0], (uint32_t)a0.x, acc);
      acc = dp4a_ss(w.qs[1], (uint32_t)a0.y, acc);
      acc = dp4a_ss(w.qs[2], (uint32_t)a0.z, acc);
      acc = dp4a_ss(w.qs[3], (uint32_t)a0.w, acc);
      acc = dp4a_ss(w.qs[4], (uint32_t)a1.x, acc);
      acc = dp4a_ss(w.qs[5], (uint32_t)a1.y, acc);
      acc = dp4a_ss(w.qs[6], (uint32_t)a1.z, acc);
      acc = dp4a_ss(w.qs[7], (uint32_t)a1.w, acc);
    }
    const float isum = __fsub_rn(__int_as_float(acc), kMagicF);  // exact
    const float s = __fmul_rn(f16_bits_to_f32(d16), ad[b]);
    sum = __fadd_rn(sum, __fmul_rn(isum, s));
  }
  return sum;
}

// Bias folded into each dp4a chain: the float-conversion magic, and for Q4_0
// the "-8" nibble offset times the activation block's q sum.
template <int WT>
__device__ __forceinline__ int32_t act_bias(int32_t qsum) {
  return WT == kQ4_0 ? kMagicI - 8 * qsum : kMagicI;
}

// ---------------------------------------------------------------------------
// Gate/up + GeGLU.  grid (I/32, E); CTA (tile, e) streams gate rows
// [32*tile, 32*tile+32) and the matching up rows of expert e once (two bulk
// copies), then runs them against every token routed to e, `tok_chunk` tokens
// at a time.  act[(sorted position) * I + row] = gelu(gate) * up.
// ---------------------------------------------------------------------------
constexpr int kGateUpThreads = 256;
constexpr int kTileRows = 32;

struct GateUpSmem {
  size_t w_off, xq_off, xd_off, xb_off, res_off, total;
};

__host__ __device__ inline GateUpSmem gate_up_smem_layout(int wtype, int H, int tok_chunk) {
  GateUpSmem L;
  const size_t rowb = (size_t)(H / 32) * block_bytes(wtype);
  size_t off = 16;  // mbarrier
  L.w_off = off;
  off += 2 * kTileRows * rowb + 16;
  off = (off + 15) & ~(size_t)15;
  L.xq_off = off;
  off += (size_t)tok_chunk * H;
  L.xd_off = off;
  off += (size_t)tok_chunk * (H / 32) * 4;
  L.xb_off = off;
  off += (size_t)tok_chunk * (H / 32) * 4;
  L.res_off = off;
  off += (size_t)tok_chunk * 2 * kTileRows * 4;
  L.total = off;
  return L;
}

template <int WT>
__global__ void __launch_bounds__(kGateUpThreads)
    gate_up_kernel(const uint8_t* __restrict__ gate_up, const int32_t* __restrict__ cnt,
                   const int32_t* __restrict__ poff, const int32_t* __restrict__ sorted,
                   const int8_t* __restrict__ xq, const float* __restrict__ xd, const int32_t* __restrict__ xsum,
                   float* __restrict__ act, int H, int I, int K, int tok_chunk, int* __restrict__ err) {
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.y, tile = blockIdx.x;
  const int beg = poff[e], n_e = cnt[e];
  if (n_e <= 0) return;
  extern __shared__ __align__(128) uint8_t smem[];
  const GateUpSmem L = gate_up_smem_layout(WT, H, tok_chunk);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint8_t* wsm = smem + L.w_off;
  int8_t* xq_s = reinterpret_cast<int8_t*>(smem + L.xq_off);
  float* xd_s = reinterpret_cast<float*>(smem + L.xd_off);
  int32_t* xb_s = reinterpret_cast<int32_t*>(smem + L.xb_off);
  float* res = reinterpret_cast<float*>(smem + L.res_off);

  const int nb = H / 32;
  const size_t rowb = (size_t)nb * block_bytes(WT);
  const uint32_t half_bytes = (uint32_t)(kTileRows * rowb);
  const uint8_t* gsrc = gate_up + ((size_t)e * 2 * I + (size_t)tile * kTileRows) * rowb;
  const uint8_t* usrc = gate_up + ((size_t)e * 2 * I + I + (size_t)tile * kTileRows) * rowb;
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, 2 * half_bytes);
    bulk_g2s(wsm, gsrc, half_bytes, bar);
    bulk_g2s(wsm + half_bytes, usrc, half_bytes, bar);
  }

  bool weights_ready = false;
  for (int c0 = 0; c0 < n_e; c0 += tok_chunk) {
    const int nc = min(tok_chunk, n_e - c0);
    // Stage the chunk's quantised activations (16-byte vectors).
    const int vec_per_tok = H / 16;
    for (int i = tid; i < nc * vec_per_tok; i += blockDim.x) {
      const int j = i / vec_per_tok, v = i % vec_per_tok;
      const int t = sorted[beg + c0 + j] / K;
      reinterpret_cast<int4*>(xq_s + (size_t)j * H)[v] = reinterpret_cast<const int4*>(xq + (size_t)t * H)[v];
    }
    for (int i = tid; i < nc * nb; i += blockDim.x) {
      const int j = i / nb, b = i % nb;
      const int t = sorted[beg + c0 + j] / K;
      xd_s[j * nb + b] = xd[(size_t)t * nb + b];
      xb_s[j * nb + b] = act_bias<WT>(xsum[(size_t)t * nb + b]);
    }
    __syncthreads();
    if (!weights_ready) {
      if (!mbar_wait_bounded(bar, 0, err)) {
        // The copy never completed: leave without touching the weights.
        return;
      }
      weights_ready = true;
    }
    // (row, token) chains: rho < 32 gate rows, rho >= 32 up rows.
    const int rho = tid & (2 * kTileRows - 1);
    for (int j = tid / (2 * kTileRows); j < nc; j += kGateUpThreads / (2 * kTileRows)) {
      res[j * 2 * kTileRows + rho] =
          row_dot_chain<WT>(wsm + (size_t)rho * rowb, nb, xq_s + (size_t)j * H, xd_s + j * nb, xb_s + j * nb);
    }
    __syncthreads();
    for (int i = tid; i < nc * kTileRows; i += blockDim.x) {
      const int j = i / kTileRows, r = i % kTileRows;
      const float g = res[j * 2 * kTileRows + r];
      const float u = res[j * 2 * kTileRows + kTileRows + r];
      act[(size_t)(beg + c0 + j) * I + tile * kTileRows + r] = __fmul_rn(gelu_approx(g), u);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Down.  grid (H/32, E); CTA (tile, e) streams 32 down rows of expert e once,
// re-quantises the act rows of the expert's tokens to Q8_0 in shared memory
// (ops.rs:175-177) and writes ydown[(sorted position) * H + row].
// ---------------------------------------------------------------------------
constexpr int kDownThreads = 256;

struct DownSmem {
  size_t w_off, xq_off, xd_off, xb_off, total;
};

__host__ __device__ inline DownSmem down_smem_layout(int wtype, int I, int tok_chunk) {
  DownSmem L;
  const size_t rowb = (size_t)(I / 32) * block_bytes(wtype);
  size_t off = 16;
  L.w_off = off;
  off += kTileRows * rowb + 16;
  off = (off + 15) & ~(size_t)15;
  L.xq_off = off;
  off += (size_t)tok_chunk * I;
  L.xd_off = off;
  off += (size_t)tok_chunk * (I / 32) * 4;
  L.xb_off = off;
  off += (size_t)tok_chunk * (I / 32) * 4;
  L.total = off;
  return L;
}

template <int WT>
__global__ void __launch_bounds__(kDownThreads)
    down_kernel(const uint8_t* __restrict__ down, const int32_t* __restrict__ cnt, const int32_t* __restrict__ poff,
                const float* __restrict__ act, float* __restrict__ ydown, int H, int I, int tok_chunk,
                int* __restrict__ err) {
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.y, tile = blockIdx.x;
  const int beg = poff[e], n_e = cnt[e];
  if (n_e <= 0) return;
  extern __shared__ __align__(128) uint8_t smem[];
  const DownSmem L = down_smem_layout(WT, I, tok_chunk);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint8_t* wsm = smem + L.w_off;
  int8_t* xq_s = reinterpret_cast<int8_t*>(smem + L.xq_off);
  float* xd_s = reinterpret_cast<float*>(smem + L.xd_off);
  int32_t* xb_s = reinterpret_cast<int32_t*>(smem + L.xb_off);

  const int nb = I / 32;
  const size_t rowb = (size_t)nb * block_bytes(WT);
  const uint32_t bytes = (uint32_t)(kTileRows * rowb);
  const uint8_t* src = down + ((size_t)e * H + (size_t)tile * kTileRows) * rowb;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(wsm, src, bytes, bar);
  }
  bool weights_ready = false;
  for (int c0 = 0; c0 < n_e; c0 += tok_chunk) {
    const int nc = min(tok_chunk, n_e - c0);
    // Re-quantise act rows to Q8_0, one warp per 32-element block.
    for (int blk = warp; blk < nc * nb; blk += kDownThreads / 32) {
      const int j = blk / nb, b = blk % nb;
      const float v = act[(size_t)(beg + c0 + j) * I + b * 32 + lane];
      int32_t qsum_dummy;
      quantize_block_warp(v, xq_s + (size_t)j * I + b * 32, xd_s + j * nb + b, &qsum_dummy, nullptr);
      if (lane == 0) xb_s[j * nb + b] = act_bias<WT>(qsum_dummy);
    }
    __syncthreads();
    if (!weights_ready) {
      if (!mbar_wait_bounded(bar, 0, err)) return;
      weights_ready = true;
    }
    const int rho = tid & (kTileRows - 1);
    for (int j = tid / kTileRows; j < nc; j += kDownThreads / kTileRows) {
      ydown[(size_t)(beg + c0 + j) * H + tile * kTileRows + rho] =
          row_dot_chain<WT>(wsm + (size_t)rho * rowb, nb, xq_s + (size_t)j * I, xd_s + j * nb, xb_s + j * nb);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Combine (model.rs:2163-2165): out[t,i] = sum over k ascending of
// (alpha_k * down_k[i]) * scale[e_k], starting from 0, skipped slots left out.
// ---------------------------------------------------------------------------
__global__ void combine_kernel(const float* __restrict__ ydown, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ ids, const float* __restrict__ probs,
                               const float* __restrict__ down_scale, float* __restrict__ out, int H, int K, int T) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T || i >= H) return;
  float o = 0.f;
  for (int k = 0; k < K; ++k) {
    const int p = pos[t * K + k];
    if (p < 0) continue;
    const float alpha = probs[t * K + k];
    const float scale = down_scale ? down_scale[ids[t * K + k]] : 1.0f;
    o = __fadd_rn(o, __fmul_rn(__fmul_rn(alpha, ydown[(size_t)p * H + i]), scale));
  }
  out[(size_t)t * H + i] = o;
}

// Combine after a speculative dispatch: the same sum, each slot's expert
// found among the token's C candidates (their positions in pos[t*C + j]).
__global__ void combine_spec_kernel(const float* __restrict__ ydown, const int32_t* __restrict__ pos,
                                    const int32_t* __restrict__ cand, const int32_t* __restrict__ ids,
                                    const float* __restrict__ probs, const float* __restrict__ down_scale,
                                    float* __restrict__ out, int H, int K, int C, int T, int* __restrict__ err) {
  __shared__ int s_p[kMaxCandidates];
  __shared__ float s_f[kMaxCandidates];
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  if (threadIdx.x < K) {
    const int k = threadIdx.x, id = ids[t * K + k];
    const float alpha = probs[t * K + k];
    int p = -1;
    if (alpha > 0.0001f) {
      for (int j = 0; j < C; ++j)
        if (cand[t * C + j] == id && pos[t * C + j] >= 0) p = pos[t * C + j];
      if (p < 0 && blockIdx.x == 0) set_error(err, kDevBadExpert);
    }
    s_p[k] = p;
    s_f[k] = p >= 0 && down_scale ? down_scale[id] : 1.0f;
  }
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H) return;
  float o = 0.f;
  for (int k = 0; k < K; ++k) {
    const int p = s_p[k];
    if (p < 0) continue;
    o = __fadd_rn(o, __fmul_rn(__fmul_rn(probs[t * K + k], ydown[(size_t)p * H + i]), s_f[k]));
  }
  out[(size_t)t * H + i] = o;
}

// 1 / sqrt(mean(row^2) + eps) with the reference's rounding (ops.rs:29-34):
// squares summed in index order in f32 by one thread, over a row staged in
// shared memory (H a multiple of 4 takes float4 loads; the order is the same).
__device__ __forceinline__ float rms_scale_seq(const float* row, int H, float eps) {
  float s = 0.f;
  int i = 0;
  if ((H & 3) == 0) {
#pragma unroll 8
    for (; i < H; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(row + i);
      s = __fadd_rn(s, __fmul_rn(v.x, v.x));
      s = __fadd_rn(s, __fmul_rn(v.y, v.y));
      s = __fadd_rn(s, __fmul_rn(v.z, v.z));
      s = __fadd_rn(s, __fmul_rn(v.w, v.w));
    }
  }
  for (; i < H; ++i) s = __fadd_rn(s, __fmul_rn(row[i], row[i]));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), eps)));
}

// Row kernels (FFN prologue / epilogue, RMS norm): one CTA of kRowThreads
// threads per row.  The row is staged in shared memory, one thread runs each
// sequential sum of squares over it (the order decides the rounding), and all
// threads do the elementwise work, four elements at a time when `vec` (H a
// multiple of 4 and every row pointer 16-byte aligned).
constexpr int kRowThreads = 128;

// Four consecutive elements of an optional weight (absent: 1).
__device__ __forceinline__ float4 ld4w(const float* w, int i) {
  return w ? *reinterpret_cast<const float4*>(w + i) : make_float4(1.f, 1.f, 1.f, 1.f);
}
__device__ __forceinline__ float4 ld4(const float* p, int i) { return *reinterpret_cast<const float4*>(p + i); }
__device__ __forceinline__ void st4(float* p, int i, float4 v) { *reinterpret_cast<float4*>(p + i) = v; }
__device__ __forceinline__ float4 mul4(float4 a, float4 b) {
  return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}
__device__ __forceinline__ float4 mul4s(float4 a, float s) {
  return make_float4(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s), __fmul_rn(a.w, s));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

__device__ __forceinline__ void stage_row(float* dst, const float* src, int H, bool vec) {
  if (vec) {
    for (int i = 4 * threadIdx.x; i < H; i += 4 * kRowThreads) st4(dst, i, ld4(src, i));
  } else {
    for (int i = threadIdx.x; i < H; i += kRowThreads) dst[i] = src[i];
  }
}

// FFN prologue of a Gemma-4 MoE layer (model.rs:1719-1784; the reference's
// GPU form is rust_cuda_prepare_ffn_f32, cuda_ptx/kernels.rs:987-1033, whose
// arguments it takes).  Per row, with the reference's CPU roundings:
//   res      = hidden + (attn * s_a) * post_attn_norm   (attn absent: hidden)
//   x_shared = (res * s) * ffn_norm             (shared dense MLP input)
//   x_moe    = (res * s) * pre_ffw_norm_2       (the experts' input)
//   router_x = ((res * s) * (1/sqrt(H))) * router_scale   (router input)
// s_a, s the rms scales of attn and res (one sum of squares serves all three
// norms).  Outputs optional, a missing weight meaning 1.
__global__ void __launch_bounds__(kRowThreads, 4)
    ffn_prologue_kernel(const float* __restrict__ hidden, const float* __restrict__ attn,
                        const float* __restrict__ pan, const float* __restrict__ ffn_norm,
                        const float* __restrict__ pre_norm2, const float* __restrict__ gis,
                        float* __restrict__ attn_res, float* __restrict__ x_shared, float* __restrict__ x_moe,
                        float* __restrict__ router_x, int H, float eps, bool vec) {
  extern __shared__ __align__(16) float row[];
  __shared__ float s_scale;
  pdl_trigger();
  pdl_wait();
  const size_t o = (size_t)blockIdx.x * H;
  const int step = vec ? 4 * kRowThreads : kRowThreads, i0 = vec ? 4 * threadIdx.x : threadIdx.x;
  if (attn) {
    stage_row(row, attn + o, H, vec);
    __syncthreads();
    if (threadIdx.x == 0) s_scale = rms_scale_seq(row, H, eps);
    __syncthreads();
    const float sa = s_scale;
    for (int i = i0; i < H; i += step) {
      if (vec) {
        st4(row, i, add4(ld4(hidden + o, i), mul4(mul4s(ld4(row, i), sa), ld4w(pan, i))));
      } else {
        float v = __fmul_rn(row[i], sa);
        if (pan) v = __fmul_rn(v, pan[i]);
        row[i] = __fadd_rn(hidden[o + i], v);
      }
    }
  } else {
    stage_row(row, hidden + o, H, vec);
  }
  __syncthreads();
  if (threadIdx.x == 0) s_scale = rms_scale_seq(row, H, eps);
  __syncthreads();
  const float sc = s_scale, inv_sqrt = __fdiv_rn(1.0f, __fsqrt_rn((float)H));
  for (int i = i0; i < H; i += step) {
    if (vec) {
      const float4 r0 = ld4(row, i), v = mul4s(r0, sc);
      if (attn_res) st4(attn_res + o, i, r0);
      if (x_shared) st4(x_shared + o, i, mul4(v, ld4w(ffn_norm, i)));
      if (x_moe) st4(x_moe + o, i, mul4(v, ld4w(pre_norm2, i)));
      if (router_x) st4(router_x + o, i, mul4(mul4s(v, inv_sqrt), ld4w(gis, i)));
    } else {
      const float r0 = row[i], v = __fmul_rn(r0, sc);
      if (attn_res) attn_res[o + i] = r0;
      if (x_shared) x_shared[o + i] = ffn_norm ? __fmul_rn(v, ffn_norm[i]) : v;
      if (x_moe) x_moe[o + i] = pre_norm2 ? __fmul_rn(v, pre_norm2[i]) : v;
      if (router_x) {
        const float r = __fmul_rn(v, inv_sqrt);
        router_x[o + i] = gis ? __fmul_rn(r, gis[i]) : r;
      }
    }
  }
}

// FFN epilogue (model.rs:2176-2196; rust_cuda_finish_ffn_f32,
// cuda_ptx/kernels.rs:1036-1083):
//   mlp_out = rms_norm(mlp_raw, post_ffw_norm_1)   (mlp_raw may be absent: 0)
//   moe_out = rms_norm(moe_raw, post_ffw_norm_2)
//   hidden  = (attn_res + rms_norm(mlp_out + moe_out, post_ffw_norm)) * out_scale
// The two first sums of squares run in two warps at once, the third after
// them.  Shared memory: two rows.
__global__ void __launch_bounds__(kRowThreads, 4)
    ffn_epilogue_kernel(const float* attn_res, const float* __restrict__ mlp_raw, const float* __restrict__ moe_raw,
                        const float* __restrict__ post1, const float* __restrict__ post2,
                        const float* __restrict__ post, float out_scale, float* hidden, int H, float eps, bool vec) {
  extern __shared__ __align__(16) float rows_s[];
  __shared__ float s_sc[3];
  pdl_trigger();
  pdl_wait();
  const size_t o = (size_t)blockIdx.x * H;
  float* ma = rows_s;  // mlp row, then the combined row
  float* mo = ma + H;  // moe row
  const int step = vec ? 4 * kRowThreads : kRowThreads, i0 = vec ? 4 * threadIdx.x : threadIdx.x;
  if (mlp_raw) {
    stage_row(ma, mlp_raw + o, H, vec);
  } else {
    for (int i = threadIdx.x; i < H; i += kRowThreads) ma[i] = 0.f;
  }
  stage_row(mo, moe_raw + o, H, vec);
  __syncthreads();
  if (threadIdx.x == 0) s_sc[0] = rms_scale_seq(ma, H, eps);
  if (threadIdx.x == 32) s_sc[1] = rms_scale_seq(mo, H, eps);
  __syncthreads();
  const float s1 = s_sc[0], s2 = s_sc[1];
  for (int i = i0; i < H; i += step) {
    if (vec) {
      st4(ma, i, add4(mul4(mul4s(ld4(ma, i), s1), ld4w(post1, i)), mul4(mul4s(ld4(mo, i), s2), ld4w(post2, i))));
    } else {
      float a = __fmul_rn(ma[i], s1);
      if (post1) a = __fmul_rn(a, post1[i]);
      float b = __fmul_rn(mo[i], s2);
      if (post2) b = __fmul_rn(b, post2[i]);
      ma[i] = __fadd_rn(a, b);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) s_sc[2] = rms_scale_seq(ma, H, eps);
  __syncthreads();
  const float s3 = s_sc[2];
  for (int i = i0; i < H; i += step) {
    if (vec) {
      const float4 v = mul4(mul4s(ld4(ma, i), s3), ld4w(post, i));
      const float4 r = add4(ld4(attn_res + o, i), v);
      st4(hidden + o, i, mul4s(r, out_scale));
    } else {
      float v = __fmul_rn(ma[i], s3);
      if (post) v = __fmul_rn(v, post[i]);
      hidden[o + i] = __fmul_rn(__fadd_rn(attn_res[o + i], v), out_scale);
    }
  }
}

// RMS normalisation of T rows of H (ops.rs:24-49): sum_sq accumulated in
// index order in f32 (x*x rounded, then added), mean = sum_sq / H,
// scale = 1 / sqrt(mean + eps), out = (x * scale) * w.
__global__ void __launch_bounds__(kRowThreads, 4)
    rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out, int H,
                    float eps, bool vec) {
  extern __shared__ __align__(16) float row[];
  __shared__ float s_scale;
  pdl_trigger();
  pdl_wait();
  const size_t o = (size_t)blockIdx.x * H;
  stage_row(row, x + o, H, vec);
  __syncthreads();
  if (threadIdx.x == 0) s_scale = rms_scale_seq(row, H, eps);
  __syncthreads();
  const float sc = s_scale;
  if (vec) {
    for (int i = 4 * threadIdx.x; i < H; i += 4 * kRowThreads) st4(out + o, i, mul4(mul4s(ld4(row, i), sc), ld4w(w, i)));
  } else {
    for (int i = threadIdx.x; i < H; i += kRowThreads) {
      const float v = __fmul_rn(row[i], sc);
      out[o + i] = w ? __fmul_rn(v, w[i]) : v;
    }
  }
}

__global__ void geglu_kernel(const float* __restrict__ gate, const float* __restrict__ up, float* __restrict__ out,
                             long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = __fmul_rn(gelu_approx(gate[i]), up[i]);
}

}  // namespace mrml

// ------------------------------------------------------------ launchers ---
namespace mrml {

static int grid_for_blocks(long long warps_needed) {
  long long g = (warps_needed + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t launch_quantize_rows(const float* x, int8_t* xq, float* xd, int32_t* xsum, long long n_blocks,
                                 cudaStream_t s) {
  return launch_pdl(quantize_rows_kernel, dim3(grid_for_blocks(n_blocks)), dim3(256), 0, s, x, xq, xd, xsum, n_blocks);
}

cudaError_t launch_geglu(const float* gate, const float* up, float* out, long long n, cudaStream_t s) {
  long long g = (n + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  geglu_kernel<<<(int)(g < 1 ? 1 : g), 256, 0, s>>>(gate, up, out, n);
  return cudaPeekAtLastError();
}

// Rows up to 200 KiB of shared memory per CTA (one row; two for the
// epilogue, which the caller asks for as 2 * H).
int rms_norm_rows_per_cta(int H) { return H > 0 && (size_t)H * 4 <= 200 * 1024 ? 1 : 0; }

namespace {
bool vec_ok(int H, std::initializer_list<const void*> ptrs) {
  if (H % 4 != 0) return false;
  for (const void* p : ptrs)
    if (((uintptr_t)p & 15) != 0) return false;
  return true;
}
}  // namespace

cudaError_t launch_rms_norm(const float* x, const float* w, float* out, int H, int T, float eps, cudaStream_t s) {
  static SmemOptIn cache;
  const size_t smem = (size_t)H * 4;
  const cudaError_t st = ensure_smem(rms_norm_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  return launch_pdl(rms_norm_kernel, dim3(T), dim3(kRowThreads), smem, s, x, w, out, H, eps, vec_ok(H, {x, w, out}));
}

// The routing of a dense FFN run as one expert: every token's one slot goes
// to expert 0 with weight 1 (so the combine's (1 * y) * 1 is y itself).
__global__ void dense_routing_kernel(int32_t* __restrict__ ids, float* __restrict__ probs, int T) {
  pdl_trigger();
  pdl_wait();
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    ids[t] = 0;
    probs[t] = 1.0f;
  }
}

cudaError_t launch_dense_routing(int32_t* ids, float* probs, int T, cudaStream_t s) {
  return launch_pdl(dense_routing_kernel, dim3(std::min(148, (T + 255) / 256)), dim3(256), 0, s, ids, probs, T);
}

cudaError_t launch_ffn_prologue(const float* hidden, const float* attn, const float* pan, const float* ffn_norm,
                                const float* pre_norm2, const float* gis, float* attn_res, float* x_shared,
                                float* x_moe, float* router_x, int H, int T, float eps, cudaStream_t s) {
  static SmemOptIn cache;
  const size_t smem = (size_t)H * 4;
  const cudaError_t st = ensure_smem(ffn_prologue_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  const bool vec = vec_ok(H, {hidden, attn, pan, ffn_norm, pre_norm2, gis, attn_res, x_shared, x_moe, router_x});
  return launch_pdl(ffn_prologue_kernel, dim3(T), dim3(kRowThreads), smem, s, hidden, attn, pan, ffn_norm, pre_norm2,
                    gis, attn_res, x_shared, x_moe, router_x, H, eps, vec);
}

cudaError_t launch_ffn_epilogue(const float* attn_res, const float* mlp_raw, const float* moe_raw, const float* post1,
                                const float* post2, const float* post, float out_scale, float* hidden, int H, int T,
                                float eps, cudaStream_t s) {
  static SmemOptIn cache;
  const size_t smem = (size_t)2 * H * 4;
  const cudaError_t st = ensure_smem(ffn_epilogue_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  const bool vec = vec_ok(H, {attn_res, mlp_raw, moe_raw, post1, post2, post, hidden});
  return launch_pdl(ffn_epilogue_kernel, dim3(T), dim3(kRowThreads), smem, s, attn_res, mlp_raw, moe_raw, post1,
                    post2, post, out_scale, hidden, H, eps, vec);
}

cudaError_t launch_quantize_gguf(int wtype, const float* x, uint8_t* dst, long long n_blocks, cudaStream_t s) {
  if (wtype == kQ8_0)
    quantize_q8_0_gguf_kernel<<<grid_for_blocks(n_blocks), 256, 0, s>>>(x, dst, n_blocks);
  else
    quantize_q4_0_gguf_kernel<<<grid_for_blocks(n_blocks), 256, 0, s>>>(x, dst, n_blocks);
  return cudaPeekAtLastError();
}

bool dispatch_topk_supported(int E, int K, int T) {
  return E >= 1 && E <= 256 && K >= 1 && K <= kMaxCandidates && K <= E && T >= 1 && T <= kDispatchTopkMaxTokens;
}

cudaError_t launch_dispatch(const int32_t* ids, const float* probs, int n_pairs, int E, int e_first, int e_total,
                            int32_t* cnt, int32_t* poff,
                            int32_t* pair_at, int32_t* pos, int4* units_gu, int4* units_dn, int* n_units,
                            int NT_gu, int NT_dn, int mt_gu, int rows_gu, int mt_dn, int* err, cudaStream_t s,
                            const float* logits, int K, int32_t* ids_out, float* probs_out, int32_t* chunk_cnt,
                            const SpecRoute* spec) {
  SpecRoute sp{};
  if (spec) {
    // speculative selection: n_pairs = T * C candidate slots
    sp = *spec;
    if (logits || !sp.lo || !sp.hi || !sp.W || !sp.x || sp.C < sp.K || sp.C > E || n_pairs % sp.C != 0 ||
        !dispatch_topk_supported(E, sp.K, n_pairs / sp.C) || !ids_out || !probs_out || e_first != 0 ||
        e_total != E)
      return cudaErrorInvalidValue;
  }
  if (logits && (!dispatch_topk_supported(E, K, n_pairs / (K > 0 ? K : 1)) || n_pairs % K != 0 || !ids_out ||
                 !probs_out))
    return cudaErrorInvalidValue;
  // The kernel reads ids and probs through the same pointers it writes them
  // with in the fused mode; otherwise it only reads them.
  const bool writes = logits || sp.lo;
  int32_t* idp = writes ? ids_out : const_cast<int32_t*>(ids);
  float* prp = writes ? probs_out : const_cast<float*>(probs);
  // the counting sort's arrays (4 [E] + [32][E+1] ints), then the selection's
  // slots ([32 warps][K] ids and values; by rank, [T][E] logits and [T][K] slots)
  const size_t T_sel = (size_t)n_pairs / (K > 0 ? K : 1);
  const size_t sel = sp.lo ? 64 * (size_t)sp.K
                    : !logits ? 0
                    : T_sel * E <= (size_t)kDispatchRankSelectMax ? T_sel * (E + 2 * K)
                                                                   : 64 * (size_t)K;
  const size_t smem = (size_t)(4 * E + 32 * (E + 1)) * 4 + sel * 4;
  static SmemOptIn dispatch_cache;
  {
    const cudaError_t st = ensure_smem(dispatch_kernel, smem, dispatch_cache);
    if (st != cudaSuccess) return st;
  }
  if (n_pairs <= kDispatchSmallPairs && K > 0 && (!logits || (n_pairs / K) * E <= kDispatchRankSelectMax)) {
    const size_t ssmem = logits ? (size_t)(n_pairs / K) * E * 4 : 0;
    return launch_pdl(dispatch_small_kernel, dim3(1), dim3(kDispatchSmallThreads), ssmem, s, idp, prp, n_pairs, E,
                      e_first, e_total, cnt, poff, pair_at, pos, units_gu, units_dn, n_units, NT_gu, NT_dn, mt_gu,
                      rows_gu, mt_dn, err, logits, K, sp);
  }
  if (!writes && chunk_cnt && n_pairs > kDispatchChunkedMin) {
    const int nchunks = (n_pairs + kDispatchThreads - 1) / kDispatchThreads;
    cudaError_t st = launch_pdl(dispatch_count_kernel, dim3(nchunks), dim3(kDispatchThreads), (size_t)E * 4, s, ids,
                                probs, n_pairs, E, e_first, e_total, chunk_cnt, err);
    if (st != cudaSuccess) return st;
    const size_t lsmem = (size_t)(4 + kLayoutTile) * E * 4;
    static SmemOptIn layout_cache;
    st = ensure_smem(dispatch_layout_kernel, lsmem, layout_cache);
    if (st != cudaSuccess) return st;
    st = launch_pdl(dispatch_layout_kernel, dim3(1), dim3(kDispatchThreads), lsmem, s, chunk_cnt,
                    nchunks, E, cnt, poff, pair_at, units_gu, units_dn, n_units, NT_gu, NT_dn, mt_gu, rows_gu, mt_dn);
    if (st != cudaSuccess) return st;
    return launch_pdl(dispatch_scatter_kernel, dim3(nchunks), dim3(kDispatchThreads), (size_t)32 * E * 4, s, ids,
                      probs, n_pairs, E, e_first, e_total, (const int32_t*)chunk_cnt, (const int32_t*)poff, pair_at,
                      pos);
  }
  cudaError_t st = launch_pdl(dispatch_kernel, dim3(1), dim3(kDispatchThreads), smem, s, idp, prp, n_pairs, E, e_first,
                              e_total, cnt, poff, pair_at, pos, units_gu, units_dn, n_units, NT_gu, NT_dn, mt_gu,
                              rows_gu, mt_dn, err, logits, K, sp);
  if (st != cudaSuccess) return st;
  return cudaPeekAtLastError();
}

cudaError_t launch_gather_groups(int wtype, const int8_t* xq, const float* xd, const int32_t* xsum,
                                 const int32_t* pair_at, const int32_t* poff_end, int H, int K, int npad, int8_t* bq,
                                 int2* bsc, cudaStream_t s) {
  const long long warps = (long long)(npad / 8) * (H / 32);  // upper bound; the kernel reads the count
  return launch_pdl(gather_groups_kernel, dim3(grid_for_blocks(warps)), dim3(256), 0, s, xq, xd, xsum, pair_at,
                    poff_end, H, K, wtype == kQ4_0 ? 1 : 0, npad, bq, bsc);
}

cudaError_t launch_quantize_scatter(int wtype, const float* x, const int32_t* pos, int T, int H, int K, int npad,
                                    bool group_major, int8_t* bq, int2* bsc, cudaStream_t s) {
  const long long warps = (long long)T * (H / 32);
  const int gm = group_major ? 1 : 0;
  if (wtype == kQ4_0)
    return launch_pdl(quantize_scatter_kernel<1>, dim3(grid_for_blocks(warps)), dim3(256), 0, s, x, pos, T, H, K, npad,
                      gm, bq, bsc);
  return launch_pdl(quantize_scatter_kernel<0>, dim3(grid_for_blocks(warps)), dim3(256), 0, s, x, pos, T, H, K, npad, gm,
                    bq, bsc);
}

constexpr size_t kMaxSmem = 227 * 1024;

int gate_up_tok_chunk(int wtype, int H) {
  for (int c = 16; c >= 1; c >>= 1)
    if (gate_up_smem_layout(wtype, H, c).total <= kMaxSmem) return c;
  return 0;
}

int down_tok_chunk(int wtype, int I) {
  for (int c = 16; c >= 1; c >>= 1)
    if (down_smem_layout(wtype, I, c).total <= kMaxSmem) return c;
  return 0;
}

cudaError_t launch_gate_up(int wtype, const uint8_t* gate_up, const int32_t* cnt, const int32_t* poff,
                           const int32_t* sorted, const int8_t* xq, const float* xd, const int32_t* xsum, float* act,
                           int H, int I, int E, int K, int* err, cudaStream_t s) {
  const int chunk = gate_up_tok_chunk(wtype, H);
  const size_t smem = gate_up_smem_layout(wtype, H, chunk).total;
  const dim3 grid(I / kTileRows, E);
  if (wtype == kQ4_0) {
    cudaError_t st = cudaFuncSetAttribute(gate_up_kernel<kQ4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
    gate_up_kernel<kQ4_0><<<grid, kGateUpThreads, smem, s>>>(gate_up, cnt, poff, sorted, xq, xd, xsum, act, H, I, K,
                                                             chunk, err);
  } else {
    cudaError_t st = cudaFuncSetAttribute(gate_up_kernel<kQ8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
    gate_up_kernel<kQ8_0><<<grid, kGateUpThreads, smem, s>>>(gate_up, cnt, poff, sorted, xq, xd, xsum, act, H, I, K,
                                                             chunk, err);
  }
  return cudaPeekAtLastError();
}

cudaError_t launch_down(int wtype, const uint8_t* down, const int32_t* cnt, const int32_t* poff, const float* act,
                        float* ydown, int H, int I, int E, int* err, cudaStream_t s) {
  const int chunk = down_tok_chunk(wtype, I);
  const size_t smem = down_smem_layout(wtype, I, chunk).total;
  const dim3 grid(H / kTileRows, E);
  if (wtype == kQ4_0) {
    cudaError_t st = cudaFuncSetAttribute(down_kernel<kQ4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
    down_kernel<kQ4_0><<<grid, kDownThreads, smem, s>>>(down, cnt, poff, act, ydown, H, I, chunk, err);
  } else {
    cudaError_t st = cudaFuncSetAttribute(down_kernel<kQ8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
    down_kernel<kQ8_0><<<grid, kDownThreads, smem, s>>>(down, cnt, poff, act, ydown, H, I, chunk, err);
  }
  return cudaPeekAtLastError();
}

cudaError_t launch_combine(const float* ydown, const int32_t* pos, const int32_t* ids, const float* probs,
                           const float* down_scale, float* out, int H, int K, int T, cudaStream_t s) {
  const dim3 grid((H + 255) / 256, T);
  return launch_pdl(combine_kernel, grid, dim3(256), 0, s, ydown, pos, ids, probs, down_scale, out, H, K, T);
}

cudaError_t launch_combine_spec(const float* ydown, const int32_t* pos, const int32_t* cand, const int32_t* ids,
                                const float* probs, const float* down_scale, float* out, int H, int K, int C, int T,
                                int* err, cudaStream_t s) {
  if (K > kMaxCandidates || K > 256) return cudaErrorInvalidValue;
  const dim3 grid((H + 255) / 256, T);
  return launch_pdl(combine_spec_kernel, grid, dim3(256), 0, s, ydown, pos, cand, ids, probs, down_scale, out, H, K,
                    C, T, err);
}

}  // namespace mrml
