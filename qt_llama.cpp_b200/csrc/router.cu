// router.cu — router logits, top-k and softmax for the MRML MoE layer.
//
// Reference behaviour (crates/mrml-tensor/src/model.rs:1804-1829): each logit
// is a sequential f32 dot product, x[i]*W[e,i] rounded, then added in index
// order; experts are sorted by logit descending (ties: lower expert id), the
// first K are kept and p_k = expf(l_k - l_0) / max(sum_k, 1e-6).
//
// The logits are computed exactly that way: one thread per (token, expert)
// runs the reference's chain over the row.  A chain of H dependent f32 adds
// is latency-bound (measured on B200: ~9.8 us for H = 2816, about 7 cycles
// per addition, with the products computed ahead or not), and T*E chains
// run side by side, so the logits, and with them the chosen ids, their
// order and the softmax weights, equal the reference's bit for bit at every
// size.
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace mrml {

constexpr int kRT = 4;             // tokens per logits CTA (one warp each)
constexpr int kRE = 32;            // experts per logits CTA (one lane each)
constexpr int kRK = 256;           // row elements per staged chunk
constexpr int kRPitch = kRK + 4;   // W chunk row pitch: lanes' float4 reads hit distinct banks
constexpr int kRStages = 4;        // chunks in flight: a chunk's chain (~1000 cycles) is shorter than a copy
constexpr int kTopkWarps = 8;       // tokens per top-k CTA

// grid (ceil(E / kRE), ceil(T / kRT)), block 32*kRT; lane l = expert e0 + l,
// warp w = token t0 + w, one chain per thread.  Row chunks stream through a
// ring of kRStages shared-memory buffers: Ws [kRE][kRPitch] (each lane reads
// its own row) and Xs [kRT][kRK] (a warp reads one row, broadcast).
// With `bulk` (H % 4 == 0, 16-byte aligned rows) thread 0 fills a stage with
// one bulk copy per row, completing on the stage's mbarrier; otherwise the
// CTA copies the chunk with plain loads.  Shared-memory reads bound the
// kernel (each warp reads its CTA's W chunk), so the CTA keeps few warps and
// the grid spreads over the SMs.
__global__ void __launch_bounds__(32 * kRT)
    router_logits_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits, int H,
                         int E, int T, int bulk, int* __restrict__ err) {
  extern __shared__ __align__(16) float rsm[];
  __shared__ __align__(8) uint64_t full[kRStages];
  float* Ws = rsm;                             // [kRStages][kRE][kRPitch]
  float* Xs = rsm + kRStages * kRE * kRPitch;  // [kRStages][kRT][kRK]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = blockIdx.x * kRE, t0 = blockIdx.y * kRT;
  const int ne = min(kRE, E - e0), nt = min(kRT, T - t0);
  const int nchunks = (H + kRK - 1) / kRK;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRStages; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  // Warp 0 fills a stage: lane 0 announces the bytes, then lane r copies
  // W row r and x row r, so the copies of a chunk issue together.
  auto issue = [&](int c) {
    const int st = c % kRStages, k0 = c * kRK, len = min(kRK, H - k0);
    if (lane == 0) mbar_arrive_expect_tx(&full[st], (uint32_t)((ne + nt) * len * 4));
    __syncwarp();
    if (lane < ne) bulk_g2s(Ws + (st * kRE + lane) * kRPitch, W + (size_t)(e0 + lane) * H + k0, len * 4, &full[st]);
    if (lane < nt) bulk_g2s(Xs + (st * kRT + lane) * kRK, x + (size_t)(t0 + lane) * H + k0, len * 4, &full[st]);
  };
  bool ok = true;
  if (bulk && warp == 0)
    for (int c = 0; c < kRStages - 1 && c < nchunks; ++c) issue(c);
  const bool active = warp < nt;  // warp-uniform
  float acc = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % kRStages, k0 = c * kRK, len = min(kRK, H - k0);
    float* ws = Ws + st * kRE * kRPitch;
    float* xs = Xs + st * kRT * kRK;
    if (bulk) {
      if (warp == 0 && __all_sync(0xffffffffu, ok) && c + kRStages - 1 < nchunks) issue(c + kRStages - 1);
      // A wait that gives up records the error; the CTA then stops computing
      // but keeps its barrier steps so that no thread is left waiting.
      if (ok && !mbar_wait_bounded(&full[st], (uint32_t)(c / kRStages) & 1u, err)) ok = false;
    } else {
      for (int q = threadIdx.x; q < (ne + nt) * len; q += blockDim.x) {
        const int r = q / len, i = q - r * len;
        if (r < ne)
          ws[r * kRPitch + i] = W[(size_t)(e0 + r) * H + k0 + i];
        else
          xs[(r - ne) * kRK + i] = x[(size_t)(t0 + r - ne) * H + k0 + i];
      }
      __syncthreads();
    }
    if (active && ok) {
      const float* wr = ws + lane * kRPitch;
      const float* xr = xs + warp * kRK;
      int i = 0;
      if (len == kRK) {
        // Loads of the next 32 elements are issued before the adds of the
        // current 32, so the chain never waits on shared memory.
        float4 xa[8], wa[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          xa[q] = *reinterpret_cast<const float4*>(xr + 4 * q);
          wa[q] = *reinterpret_cast<const float4*>(wr + 4 * q);
        }
#pragma unroll 1
        for (; i < kRK; i += 32) {
          float4 xb[8], wb[8];
          const int nx = i + 32 < kRK ? i + 32 : i;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            xb[q] = *reinterpret_cast<const float4*>(xr + nx + 4 * q);
            wb[q] = *reinterpret_cast<const float4*>(wr + nx + 4 * q);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            acc = __fadd_rn(acc, __fmul_rn(xa[q].x, wa[q].x));
            acc = __fadd_rn(acc, __fmul_rn(xa[q].y, wa[q].y));
            acc = __fadd_rn(acc, __fmul_rn(xa[q].z, wa[q].z));
            acc = __fadd_rn(acc, __fmul_rn(xa[q].w, wa[q].w));
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            xa[q] = xb[q];
            wa[q] = wb[q];
          }
        }
      } else {
        for (; i < len; ++i) acc = __fadd_rn(acc, __fmul_rn(xr[i], wr[i]));
      }
    }
    __syncthreads();  // the stage is refilled in the next iteration
  }
  if (!ok && bulk && threadIdx.x == 0) {
    // Let copies still in flight land before the CTA exits.
    for (int c = 0; c < nchunks; ++c) mbar_wait_bounded(&full[c % kRStages], (uint32_t)(c / kRStages) & 1u, err);
  }
  const int t = t0 + warp, e = e0 + lane;
  if (ok && t < T && e < E) logits[(size_t)t * E + e] = acc;
}

// Whole-row variant for rows that fit: the CTA (kRT warps = tokens, lanes
// 0..kRE2-1 = experts) loads its kRE2 W rows and kRT x rows with one bulk
// copy each, waits once, and runs the chains with register prefetch.  Row
// pitch H + 4 floats keeps the lanes' float4 reads on distinct banks.
constexpr int kRE2 = 16;

__host__ __device__ inline size_t router_rows_smem(int H) {
  return (size_t)(kRE2 + kRT) * (size_t)(H + 4) * sizeof(float);
}

// With prefetch_bytes > 0, the CTAs also ask the L2 for that many bytes from
// `prefetch` (split evenly, in 64 KiB bulk prefetches): the expert weights the
// next products read first, fetched while the router, dispatch and quantise
// launches leave the HBM idle.  A hint only; nothing waits for it.
__global__ void __launch_bounds__(32 * kRT)
    router_logits_rows_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                              int H, int E, int T, int* __restrict__ err, const uint8_t* prefetch,
                              size_t prefetch_bytes) {
  extern __shared__ __align__(16) float rsm[];
  __shared__ __align__(8) uint64_t full;
  const int pitch = H + 4;
  float* Ws = rsm;                 // [kRE2][pitch]
  float* Xs = rsm + kRE2 * pitch;  // [kRT][pitch]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = blockIdx.x * kRE2, t0 = blockIdx.y * kRT;
  const int ne = min(kRE2, E - e0), nt = min(kRT, T - t0);
  pdl_trigger();
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    // The router weights are not written by earlier kernels: their copies
    // start while the previous kernel finishes; the inputs wait for it.
    if (lane == 0) mbar_arrive_expect_tx(&full, (uint32_t)((ne + nt) * H * 4));
    __syncwarp();
    if (lane < ne) bulk_g2s(Ws + lane * pitch, W + (size_t)(e0 + lane) * H, H * 4, &full);
    pdl_wait();
    if (lane < nt) bulk_g2s(Xs + lane * pitch, x + (size_t)(t0 + lane) * H, H * 4, &full);
  }
  if (!mbar_wait_bounded(&full, 0, err)) {
    if (threadIdx.x == 0) mbar_wait_bounded(&full, 0, err);  // let copies in flight land
    return;
  }
  if (warp == 1 && prefetch_bytes > 0) {
    // this CTA's share of the prefetch, one 64 KiB chunk per lane at a time,
    // issued once the CTA's own rows have landed
    constexpr size_t kChunk = 64 * 1024;
    const size_t n_chunks = (prefetch_bytes + kChunk - 1) / kChunk;
    const size_t nct = (size_t)gridDim.x * gridDim.y, cta = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    for (size_t c = cta + nct * lane; c < n_chunks; c += nct * 32) {
      const size_t off = c * kChunk;
      const uint32_t bytes = (uint32_t)(prefetch_bytes - off < kChunk ? prefetch_bytes - off : kChunk);
      bulk_prefetch_l2(prefetch + off, bytes);
    }
  }
  if (warp >= nt || lane >= ne) return;
  const float* wr = Ws + lane * pitch;
  const float* xr = Xs + warp * pitch;
  float acc = 0.f;
  float4 xa[8], wa[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    xa[q] = *reinterpret_cast<const float4*>(xr + 4 * q);
    wa[q] = *reinterpret_cast<const float4*>(wr + 4 * q);
  }
  // H is a multiple of 32 here.
#pragma unroll 1
  for (int i = 0; i < H; i += 32) {
    float4 xb[8], wb[8];
    const int nx = i + 32 < H ? i + 32 : i;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      xb[q] = *reinterpret_cast<const float4*>(xr + nx + 4 * q);
      wb[q] = *reinterpret_cast<const float4*>(wr + nx + 4 * q);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      acc = __fadd_rn(acc, __fmul_rn(xa[q].x, wa[q].x));
      acc = __fadd_rn(acc, __fmul_rn(xa[q].y, wa[q].y));
      acc = __fadd_rn(acc, __fmul_rn(xa[q].z, wa[q].z));
      acc = __fadd_rn(acc, __fmul_rn(xa[q].w, wa[q].w));
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      xa[q] = xb[q];
      wa[q] = wb[q];
    }
  }
  logits[(size_t)(t0 + warp) * E + e0 + lane] = acc;
}

// Large-batch variant (many tokens): throughput rather than latency.  CTA =
// 32 experts (lanes) × 32 tokens (8 warps × 4 tokens per thread), so a W
// value read from shared memory serves 4 chains and an x value (broadcast
// in the warp) 32.  Rows stream in chunks of kTK elements through a
// kTStages ring filled with 16-byte asynchronous copies (4 per thread per
// chunk); W rows are padded so that the lanes' float4 reads hit distinct
// banks.  Needs H % 4 == 0 and 16-byte aligned rows.
constexpr int kTE = 32, kTWarps = 8, kTB = 4, kTT = kTWarps * kTB;
constexpr int kTK = 64, kTPitch = kTK + 4, kTStages = 3;
constexpr size_t kTStageFloats = (size_t)kTE * kTPitch + (size_t)kTT * kTK;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_stages() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kTStages - 1) : "memory");
}

__device__ __forceinline__ void tiled_stage(float* st, const float* __restrict__ W, const float* __restrict__ x, int H,
                                            int e0, int ne, int t0, int nt, int k0, int len) {
  float* Ws = st;
  float* Xs = st + kTE * kTPitch;
  const int pieces = len >> 2;  // float4 pieces per row
  for (int q = threadIdx.x; q < (kTE + kTT) * pieces; q += blockDim.x) {
    const int r = q / pieces, c = (q - r * pieces) << 2;
    if (r < kTE) {
      if (r < ne) cp_async16(Ws + r * kTPitch + c, W + (size_t)(e0 + r) * H + k0 + c);
    } else if (r - kTE < nt) {
      cp_async16(Xs + (r - kTE) * kTK + c, x + (size_t)(t0 + r - kTE) * H + k0 + c);
    }
  }
  cp_async_commit();  // one group per chunk, possibly empty
}

__global__ void __launch_bounds__(32 * kTWarps)
    router_logits_tiled_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ logits,
                               int H, int E, int T) {
  extern __shared__ __align__(16) float tsm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = blockIdx.x * kTE, t0 = blockIdx.y * kTT;
  const int ne = min(kTE, E - e0), nt = min(kTT, T - t0);
  const int nchunks = (H + kTK - 1) / kTK;
  pdl_trigger();
  pdl_wait();
  for (int c = 0; c < kTStages - 1; ++c) {
    if (c < nchunks)
      tiled_stage(tsm + c * kTStageFloats, W, x, H, e0, ne, t0, nt, c * kTK, min(kTK, H - c * kTK));
    else
      cp_async_commit();
  }
  float acc[kTB];
#pragma unroll
  for (int j = 0; j < kTB; ++j) acc[j] = 0.f;
  const bool active = kTB * warp < nt;  // warp-uniform
  for (int c = 0; c < nchunks; ++c) {
    const int cn = c + kTStages - 1;
    if (cn < nchunks)
      tiled_stage(tsm + (cn % kTStages) * kTStageFloats, W, x, H, e0, ne, t0, nt, cn * kTK, min(kTK, H - cn * kTK));
    else
      cp_async_commit();
    cp_async_wait_stages();
    __syncthreads();
    const float* st = tsm + (c % kTStages) * kTStageFloats;
    const float* wr = st + lane * kTPitch;
    const float* xr = st + kTE * kTPitch + kTB * warp * kTK;
    const int len = min(kTK, H - c * kTK);
    if (active) {
#pragma unroll 4
      for (int i = 0; i < len; i += 4) {
        const float4 b = *reinterpret_cast<const float4*>(wr + i);
#pragma unroll
        for (int j = 0; j < kTB; ++j) {
          const float4 a = *reinterpret_cast<const float4*>(xr + j * kTK + i);
          acc[j] = __fadd_rn(acc[j], __fmul_rn(a.x, b.x));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(a.y, b.y));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(a.z, b.z));
          acc[j] = __fadd_rn(acc[j], __fmul_rn(a.w, b.w));
        }
      }
    }
    __syncthreads();  // the stage is refilled in the next iteration
  }
  if (lane < ne) {
#pragma unroll
    for (int j = 0; j < kTB; ++j) {
      const int t = t0 + kTB * warp + j;
      if (t < T) logits[(size_t)t * E + e0 + lane] = acc[j];
    }
  }
}

struct TopkShared {
  int cand[kTopkWarps][kMaxCandidates];
  float cval[kTopkWarps][kMaxCandidates];
};

// grid ceil(T / kTopkWarps), block 32*kTopkWarps; one warp per token: the
// K best experts of the token's logits (value desc, id asc) and their
// softmax weights.
template <int PL>
__global__ void __launch_bounds__(32 * kTopkWarps)
    router_topk_kernel(const float* __restrict__ logits, int32_t* __restrict__ ids, float* __restrict__ probs, int E,
                       int K, int T) {
  __shared__ TopkShared S;
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int t = blockIdx.x * kTopkWarps + wl;
  if (t >= T) return;
  const float* lrow = logits + (size_t)t * E;
  float val[PL];
#pragma unroll
  for (int m = 0; m < PL; ++m) {
    const int e = lane + 32 * m;
    val[m] = e < E ? lrow[e] : -INFINITY;
  }
  uint32_t taken;
  warp_topk<PL>(val, E, K, S.cand[wl], S.cval[wl], taken);
  finish_token(S.cand[wl], S.cval[wl], K, K, t, ids, probs);
}

// ---------------------------------------------------------------------------
// Router logit intervals for the small-batch forward (speculative routing).
// The reference's logit is the chain s_i = fl(s_{i-1} + fl(p_i)), p_i =
// x_i * w_i, i ascending (model.rs:1804-1814).  With u = 2^-24, t = 2^-149
// and S_i the exact prefix sums, each step gives |s_i - s_{i-1} - fl(p_i)|
// <= u/(1-u) |s_i| and |fl(p_i) - p_i| <= u |p_i| + t, so
//   |s_n - S_n| <= u P + n t + u/(1-u) (sum_i |S_i| + n E_n),
// P = sum |p_i|, E_n = gamma_{n+1} (P + n t) bounding every |s_i - S_i|.
// Lane l of a warp takes a contiguous run of m = n/32 elements and sums
// fl(p_i) along it in f32 (the runs' totals r_l, prefixes q_i); a warp scan
// of the totals in f64 gives each run's offset o_l and the centre c.  Each
// f32 run sum is within G = gamma_{m+1} P + m t of the exact one, so
//   |c - S_n| <= G + n t   and   |S_i| <= |o_l| + |q_i| + 2 (G + n t),
//   sum_i |S_i| <= sum_l (m |o_l| + sum_i |q_i|) + 2 n (G + n t).
// The interval is c -/+ (both bounds), with a 1e-3 relative margin for the
// f32 sums of magnitudes (relative error below 100 u) and the evaluation,
// rounded outward to f32.
// A CTA stages kBE experts' router rows and kBT tokens' inputs in shared
// memory with bulk copies; warp w takes expert w against each token.
// ---------------------------------------------------------------------------
constexpr int kBE = 8, kBT = 4;

__host__ __device__ inline size_t router_bounds_smem(int H) { return (size_t)(kBE + kBT) * H * sizeof(float); }

__global__ void __launch_bounds__(32 * kBE)
    router_bounds_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ lo,
                         float* __restrict__ hi, int H, int E, int T, int* __restrict__ err) {
  extern __shared__ __align__(16) float bsm[];
  __shared__ __align__(8) uint64_t full;
  float* Ws = bsm;           // [kBE][H]
  float* Xs = bsm + kBE * H; // [kBT][H]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = blockIdx.x * kBE, t0 = blockIdx.y * kBT;
  const int ne = min(kBE, E - e0), nt = min(kBT, T - t0);
  pdl_trigger();
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    // the router weights are not written by earlier kernels; the inputs are
    if (lane == 0) mbar_arrive_expect_tx(&full, (uint32_t)((ne + nt) * H * 4));
    __syncwarp();
    if (lane < ne) bulk_g2s(Ws + lane * H, W + (size_t)(e0 + lane) * H, H * 4, &full);
    pdl_wait();
    if (lane < nt) bulk_g2s(Xs + lane * H, x + (size_t)(t0 + lane) * H, H * 4, &full);
  }
  if (!mbar_wait_bounded(&full, 0, err)) {
    if (threadIdx.x == 0) mbar_wait_bounded(&full, 0, err);  // let copies in flight land
    return;
  }
  if (warp >= ne) return;
  const int per = H / 32;  // H % 128 == 0: runs of a multiple of 4 elements
  const float4* wr = reinterpret_cast<const float4*>(Ws + warp * H + lane * per);
  float run[kBT], absl[kBT], absp[kBT];
#pragma unroll
  for (int j = 0; j < kBT; ++j) {
    run[j] = 0.f;
    absl[j] = 0.f;
    absp[j] = 0.f;
  }
#pragma unroll 2
  for (int q = 0; q < per / 4; ++q) {
    const float4 b = wr[q];
#pragma unroll
    for (int j = 0; j < kBT; ++j) {
      if (j < nt) {
        const float4 a = reinterpret_cast<const float4*>(Xs + j * H + lane * per)[q];
        const float p0 = __fmul_rn(a.x, b.x), p1 = __fmul_rn(a.y, b.y);
        const float p2 = __fmul_rn(a.z, b.z), p3 = __fmul_rn(a.w, b.w);
        run[j] = __fadd_rn(run[j], p0);
        absl[j] = __fadd_rn(absl[j], fabsf(run[j]));
        run[j] = __fadd_rn(run[j], p1);
        absl[j] = __fadd_rn(absl[j], fabsf(run[j]));
        run[j] = __fadd_rn(run[j], p2);
        absl[j] = __fadd_rn(absl[j], fabsf(run[j]));
        run[j] = __fadd_rn(run[j], p3);
        absl[j] = __fadd_rn(absl[j], fabsf(run[j]));
        absp[j] = __fadd_rn(absp[j], __fadd_rn(__fadd_rn(fabsf(p0), fabsf(p1)), __fadd_rn(fabsf(p2), fabsf(p3))));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kBT; ++j) {
    if (j >= nt) break;
    // exclusive scan of the runs' totals (f64): each run's offset
    const double r = (double)run[j];
    double incl = r;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const double off = incl - r;
    double sabs = (double)per * fabs(off) + (double)absl[j], sump = (double)absp[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sabs += __shfl_xor_sync(0xffffffffu, sabs, o);
      sump += __shfl_xor_sync(0xffffffffu, sump, o);
    }
    const double total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      const double u = 0x1p-24, n = (double)H, m = (double)per, t = 0x1p-149;
      const double gam_n = (n + 1.0) * u / (1.0 - (n + 1.0) * u), gam_m = (m + 1.0) * u / (1.0 - (m + 1.0) * u);
      const double g = gam_m * sump + m * t + n * t;     // run-sum error, plus the f64 scan's below it
      const double en = gam_n * (sump + n * t);
      const double sum_s = sabs + 2.0 * n * g;
      const double bnd = (u * sump + n * t + u / (1.0 - u) * (sum_s + n * en) + g) * 1.001 + 0x1p-140;
      const size_t o = (size_t)(t0 + j) * E + e0 + warp;
      lo[o] = __double2float_rd(total - bnd);
      hi[o] = __double2float_ru(total + bnd);
    }
  }
}

// ------------------------------------------------------------ launchers ---

cudaError_t launch_router_logits(const float* W, const float* x, float* logits, int H, int E, int T, int* err,
                                 cudaStream_t s, const uint8_t* prefetch, size_t prefetch_bytes) {
  static SmemOptIn cache, cache_rows, cache_tiled;
  const bool aligned = (((uintptr_t)W | (uintptr_t)x) & 15) == 0;
  // Large batches: the tiled kernel (throughput); decode batches: whole rows
  // per CTA (latency).  Measured crossover on B200 at H = 2816: ~256 tokens.
  if (aligned && H % 4 == 0 && T > 256) {
    const dim3 grid((E + kTE - 1) / kTE, (T + kTT - 1) / kTT);
    const size_t smem = kTStages * kTStageFloats * sizeof(float);
    cudaError_t st = ensure_smem(router_logits_tiled_kernel, smem, cache_tiled);
    if (st != cudaSuccess) return st;
    return launch_pdl(router_logits_tiled_kernel, grid, dim3(32 * kTWarps), smem, s, W, x, logits, H, E, T);
  }
  if (aligned && H % 32 == 0 && router_rows_smem(H) <= 227 * 1024) {
    const dim3 grid((E + kRE2 - 1) / kRE2, (T + kRT - 1) / kRT);
    const size_t smem = router_rows_smem(H);
    cudaError_t st = ensure_smem(router_logits_rows_kernel, smem, cache_rows);
    if (st != cudaSuccess) return st;
    // bulk prefetches want 16-byte addresses and sizes
    const bool pf = prefetch && ((uintptr_t)prefetch & 15) == 0 && prefetch_bytes % 16 == 0;
    return launch_pdl(router_logits_rows_kernel, grid, dim3(32 * kRT), smem, s, W, x, logits, H, E, T, err,
                      pf ? prefetch : nullptr, pf ? prefetch_bytes : (size_t)0);
  }
  const dim3 grid((E + kRE - 1) / kRE, (T + kRT - 1) / kRT);
  const bool bulk = H % 4 == 0 && (((uintptr_t)W | (uintptr_t)x) & 15) == 0;
  const size_t smem = (size_t)kRStages * (kRE * kRPitch + kRT * kRK) * sizeof(float);
  cudaError_t st = ensure_smem(router_logits_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  return launch_pdl(router_logits_kernel, grid, dim3(32 * kRT), smem, s, W, x, logits, H, E, T, bulk ? 1 : 0, err);
}

bool router_bounds_supported(const float* W, const float* x, int H) {
  return H > 0 && H % 128 == 0 && router_bounds_smem(H) <= 227 * 1024 && (((uintptr_t)W | (uintptr_t)x) & 15) == 0;
}

cudaError_t launch_router_bounds(const float* W, const float* x, float* lo, float* hi, int H, int E, int T, int* err,
                                 cudaStream_t s) {
  static SmemOptIn cache;
  const size_t smem = router_bounds_smem(H);
  const cudaError_t st = ensure_smem(router_bounds_kernel, smem, cache);
  if (st != cudaSuccess) return st;
  const dim3 grid((E + kBE - 1) / kBE, (T + kBT - 1) / kBT);
  return launch_pdl(router_bounds_kernel, grid, dim3(32 * kBE), smem, s, W, x, lo, hi, H, E, T, err);
}

cudaError_t launch_router_topk(const float* logits, int32_t* ids, float* probs, int E, int K, int T, cudaStream_t s) {
  const dim3 grid((T + kTopkWarps - 1) / kTopkWarps);
  const int block = 32 * kTopkWarps;
  if (E <= 32) return launch_pdl(router_topk_kernel<1>, grid, dim3(block), 0, s, logits, ids, probs, E, K, T);
  if (E <= 128) return launch_pdl(router_topk_kernel<4>, grid, dim3(block), 0, s, logits, ids, probs, E, K, T);
  return launch_pdl(router_topk_kernel<8>, grid, dim3(block), 0, s, logits, ids, probs, E, K, T);
}

}  // namespace mrml
