// gemm_tc.cu — grouped expert products on the 5th-generation tensor cores.
//
// One persistent kernel per product (gate/up, down).  A work unit is
// (expert e, 128 weight rows, a tile of NT token positions routed to e).
// The reference's arithmetic per weight row r and token j is
//     sum_b fl( (float)isum_b(r, j) * fl(d_w[r,b] * d_a[j,b]) )
// accumulated in block order b = 0, 1, ... (quant.rs:335-369 / 564-577).
// isum_b is an exact int32 dot of 32 int8 (or unsigned nibble) weights with
// 32 int8 activations, which is exactly one tcgen05.mma kind::i8 with K = 32.
// So each quant block is one MMA into its own TMEM accumulator, and the f32
// scale-and-accumulate runs in the epilogue warps in the reference's order.
//
// Warp roles (one CTA per SM, persistent over units):
//   warp 0       weight producer: raw GGUF weight chunks (TMA tensor-map
//                tiles, or 1-D bulk copies of whole rows)
//   warp 1       TMEM allocation; lane 0 issues the MMAs
//   warp 2       activation producer: B tiles and their scales (bulk copies)
//   warps 3..6   converters: raw Q4_0/Q8_0 bytes -> int8 A tiles in the
//                canonical no-swizzle K-major layout, f16 scales -> f32
//   warps 7..    epilogue: tcgen05.ld, block scaling, GeGLU, re-quantisation
//                of act (gate/up) or the f32 down rows (down)
// The two producers run independently, so the HBM weight stream can run as
// far ahead as its ring allows, whatever the activation ring's depth.
// Every mbarrier wait is bounded; on a timeout the CTA records the error,
// drops out of its loops, frees its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"

namespace mrml {
namespace tc {

// Pipeline helpers (Bars, bounded waits, TMA, descriptors) live in pipe.cuh.

// ------------------------------------------------------------------ kernel
template <int WQ4, int MODE, int NT>
__global__ void __launch_bounds__(32 * (kEpiWarp0 + 4 * ((NT + 31) / 32)), 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap, const Params P) {
  constexpr int BB = WQ4 ? 18 : 34;
  constexpr int NA = MODE == kGateUp ? 2 : 1;     // A tiles per block (gate, up)
  constexpr int CPB = NA * NT;                     // TMEM columns per block
  constexpr int TPW = NT < 32 ? NT : 32;           // tokens per epilogue thread
  constexpr int EW = 4 * ((NT + 31) / 32);         // epilogue warps
  constexpr uint32_t IDESC = idesc_i8(WQ4 != 0, NT, kM);
  constexpr int A_BYTES = kM * 32;                 // one A tile
  constexpr int SLOT_BYTES = NA * A_BYTES;
  constexpr int DW_BYTES = NA * kM * 4;
  constexpr int kG = NT <= 16 ? 4 : 1;             // blocks per epilogue round (decode tiles)

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  Bars* B = reinterpret_cast<Bars*>(smem);
  uint8_t* raw = smem + 1024;
  uint8_t* conv = raw + P.rs * P.raw_bytes;   // A tiles, 1024-aligned (raw_bytes multiple of 1024)
  float* dwr = reinterpret_cast<float*>(conv + P.as * SLOT_BYTES);  // weight scales, P.tb slots
  uint8_t* bsb = reinterpret_cast<uint8_t*>(dwr) + P.tb * DW_BYTES;  // B tiles + scales
  const int bs_stage = P.kcb * NT * (32 + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.rs; ++i) {
      mbar_init(&B->raw_full[i], 1);
      mbar_init(&B->raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < P.as; ++i) {
      mbar_init(&B->conv_full[i], kConvWarps);
      mbar_init(&B->conv_empty[i], 1);
    }
    for (int i = 0; i < P.tb; ++i) {
      mbar_init(&B->dw_full[i], kConvWarps);
      mbar_init(&B->dw_empty[i], EW);
    }
    for (int i = 0; i < P.bs; ++i) {
      mbar_init(&B->bs_full[i], 1);
      mbar_init(&B->bs_empty[i], EW);
    }
    for (int i = 0; i < P.tb; ++i) {
      mbar_init(&B->tmem_full[i], 1);
      mbar_init(&B->tmem_empty[i], EW);
    }
    B->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&B->tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = B->tmem_base;
  const int n_units = *P.n_units;
  const int nkc = MODE == kGateUp ? P.nb / kKC : 1;

  if (warp == 0) {
    // ----------------------------------------------------- weight producer
    if (lane == 0) {
      int rs = 0;
      uint32_t rph = 0;
      for (int u = blockIdx.x; u < n_units && !aborted(B); u += gridDim.x) {
        const int4 U = P.units[u];
        const int e = U.x, m0 = U.w;
        for (int kc = 0; kc < nkc; ++kc) {
          if (!wait_bar(&B->raw_empty[rs], rph ^ 1, B, P.err)) break;
          uint8_t* dst = raw + rs * P.raw_bytes;
          if constexpr (MODE == kGateUp) {
            mbar_arrive_expect_tx(&B->raw_full[rs], 2 * kM * kKC * BB);
            const int c0 = kc * kKC * BB / 2;  // 16-bit elements
            tma_load_3d(dst, &tmap, c0, m0, 2 * e, &B->raw_full[rs]);
            tma_load_3d(dst + kM * kKC * BB, &tmap, c0, m0, 2 * e + 1, &B->raw_full[rs]);
          } else {
            const int nrows = min(kM, P.rows - m0);
            const uint32_t bytes = (uint32_t)(nrows * P.row_bytes);
            mbar_arrive_expect_tx(&B->raw_full[rs], bytes);
            bulk_g2s(dst, P.w_raw + ((size_t)e * P.rows + m0) * P.row_bytes, bytes, &B->raw_full[rs]);
          }
          if (++rs == P.rs) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------- activation producer
    if (lane == 0) {
      int bsi = 0;
      uint32_t bph = 0;
      for (int u = blockIdx.x; u < n_units && !aborted(B); u += gridDim.x) {
        const int p0 = P.units[u].y;
        for (int kc = 0; kc < nkc; ++kc) {
          if (!wait_bar(&B->bs_empty[bsi], bph ^ 1, B, P.err)) break;
          uint8_t* bdst = bsb + bsi * bs_stage;
          const int b0 = kc * P.kcb;
          const int nblk = min(P.kcb, P.nb - b0);
          mbar_arrive_expect_tx(&B->bs_full[bsi], (uint32_t)(nblk * NT * 40));
          for (int bl = 0; bl < nblk; ++bl) {
            const int b = b0 + bl;
            bulk_g2s(bdst + bl * NT * 32, P.bq + ((size_t)b * (P.npad / 8) + p0 / 8) * 256, NT * 32, &B->bs_full[bsi]);
            bulk_g2s(bdst + P.kcb * NT * 32 + bl * NT * 8, P.bsc + (size_t)b * P.npad + p0, NT * 8, &B->bs_full[bsi]);
          }
          if (++bsi == P.bs) {
            bsi = 0;
            bph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      int as = 0, ts = 0, bsi = 0;
      uint32_t aph = 0, tph = 0, bph = 0;
      for (int u = blockIdx.x; u < n_units && !aborted(B); u += gridDim.x) {
        bool ok = true;
        for (int kc = 0; kc < nkc && ok; ++kc) {
          if (!(ok = wait_bar(&B->bs_full[bsi], bph, B, P.err))) break;
          const uint8_t* bt = bsb + bsi * bs_stage;
          const int nblk = min(P.kcb, P.nb - kc * P.kcb);
          for (int bl = 0; bl < nblk; ++bl) {
            if (!(ok = wait_bar(&B->conv_full[as], aph, B, P.err))) break;
            if (!(ok = wait_bar(&B->tmem_empty[ts], tph ^ 1, B, P.err))) break;
            fence_after();
            const uint8_t* slot = conv + as * SLOT_BYTES;
            const uint64_t bdesc = smem_desc(bt + bl * NT * 32);
            mma_i8(tmem + ts * CPB, smem_desc(slot), bdesc, IDESC);
            if constexpr (NA == 2) mma_i8(tmem + ts * CPB + NT, smem_desc(slot + A_BYTES), bdesc, IDESC);
            mma_commit(&B->conv_empty[as]);  // A slot reusable once these MMAs have read it
            mma_commit(&B->tmem_full[ts]);
            if (++as == P.as) {
              as = 0;
              aph ^= 1;
            }
            if (++ts == P.tb) {
              ts = 0;
              tph ^= 1;
            }
          }
          if (++bsi == P.bs) {
            bsi = 0;
            bph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp < kEpiWarp0) {
    // ---------------------------------------------------------- converters
    const int r = threadIdx.x - 32 * kConvWarp0;  // weight row within the tile
    int rs = 0, as = 0, ts = 0;
    uint32_t rph = 0, aph = 0, tph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok && !aborted(B); u += gridDim.x) {
      for (int kc = 0; kc < nkc && ok; ++kc) {
        if (!(ok = wait_bar(&B->raw_full[rs], rph, B, P.err))) break;
        const uint8_t* src = raw + rs * P.raw_bytes;
        if constexpr (MODE == kGateUp) {
          const uint8_t* grow = src + r * (kKC * BB);
          const uint8_t* urow = src + kM * kKC * BB + r * (kKC * BB);
#define MRML_CONV_BLOCK(BL)                                                                   \
  {                                                                                           \
    if (ok) ok = wait_bar(&B->conv_empty[as], aph ^ 1, B, P.err);                             \
    if (ok) ok = wait_bar(&B->dw_empty[ts], tph ^ 1, B, P.err);                               \
    if (ok) {                                                                                 \
      uint8_t* slot = conv + as * SLOT_BYTES;                                                 \
      float* dws = dwr + ts * (NA * kM);                                                      \
      uint32_t d16;                                                                           \
      uint32_t qs[BB == 18 ? 4 : 8];                                                          \
      uint4 lo, hi;                                                                           \
      chunk_block<BB, BL>(grow, d16, qs);                                                     \
      if constexpr (BB == 18) q4_to_a(qs, lo, hi);                                            \
      else { lo = make_uint4(qs[0], qs[1], qs[2], qs[3]); hi = make_uint4(qs[4], qs[5], qs[6], qs[7]); } \
      store_a_row(reinterpret_cast<int8_t*>(slot), r, lo, hi);                                \
      dws[r] = f16_bits_to_f32(d16);                                                          \
      chunk_block<BB, BL>(urow, d16, qs);                                                     \
      if constexpr (BB == 18) q4_to_a(qs, lo, hi);                                            \
      else { lo = make_uint4(qs[0], qs[1], qs[2], qs[3]); hi = make_uint4(qs[4], qs[5], qs[6], qs[7]); } \
      store_a_row(reinterpret_cast<int8_t*>(slot + A_BYTES), r, lo, hi);                      \
      dws[kM + r] = f16_bits_to_f32(d16);                                                     \
      fence_proxy_async();                                                                    \
      __syncwarp();                                                                           \
      if (lane == 0) {                                                                        \
        mbar_arrive(&B->conv_full[as]);                                                       \
        mbar_arrive(&B->dw_full[ts]);                                                         \
      }                                                                                       \
      if (++as == P.as) { as = 0; aph ^= 1; }                                                 \
      if (++ts == P.tb) { ts = 0; tph ^= 1; }                                                 \
    }                                                                                         \
  }
          MRML_CONV_BLOCK(0) MRML_CONV_BLOCK(1) MRML_CONV_BLOCK(2) MRML_CONV_BLOCK(3)
          MRML_CONV_BLOCK(4) MRML_CONV_BLOCK(5) MRML_CONV_BLOCK(6) MRML_CONV_BLOCK(7)
#undef MRML_CONV_BLOCK
        } else {
          const uint8_t* row = src + (size_t)r * P.row_bytes;
          for (int b = 0; b < P.nb && ok; ++b) {
            if (!(ok = wait_bar(&B->conv_empty[as], aph ^ 1, B, P.err))) break;
            if (!(ok = wait_bar(&B->dw_empty[ts], tph ^ 1, B, P.err))) break;
            uint8_t* slot = conv + as * SLOT_BYTES;
            float* dws = dwr + ts * (NA * kM);
            uint4 lo, hi;
            uint32_t d16;
            if constexpr (BB == 18) {
              const Q4Block q = load_q4_block(row + b * 18);
              d16 = q.d16;
              q4_to_a(q.qs, lo, hi);
            } else {
              const Q8Block q = load_q8_block(row + b * 34);
              d16 = q.d16;
              lo = make_uint4(q.qs[0], q.qs[1], q.qs[2], q.qs[3]);
              hi = make_uint4(q.qs[4], q.qs[5], q.qs[6], q.qs[7]);
            }
            store_a_row(reinterpret_cast<int8_t*>(slot), r, lo, hi);
            dws[r] = f16_bits_to_f32(d16);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&B->conv_full[as]);
              mbar_arrive(&B->dw_full[ts]);
            }
            if (++as == P.as) {
              as = 0;
              aph ^= 1;
            }
            if (++ts == P.tb) {
              ts = 0;
              tph ^= 1;
            }
          }
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&B->raw_empty[rs]);
        if (++rs == P.rs) {
          rs = 0;
          rph ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - kEpiWarp0;
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int j0 = (ew >> 2) * TPW;  // first token column of this warp
    int ts = 0, bsi = 0;
    uint32_t tph = 0, bph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok && !aborted(B); u += gridDim.x) {
      const int4 U = P.units[u];
      const int p0 = U.y, nvalid = U.z, m0 = U.w;
      const int nj = max(0, min(TPW, nvalid - j0));
      const int row = m0 + 32 * q + lane;
      float acc[NA][TPW];
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int j = 0; j < TPW; ++j) acc[a][j] = 0.f;
      for (int kc = 0; kc < nkc && ok; ++kc) {
        if (!(ok = wait_bar(&B->bs_full[bsi], bph, B, P.err))) break;
        const int2* sc = reinterpret_cast<const int2*>(bsb + bsi * bs_stage + P.kcb * NT * 32);
        const int nblk = min(P.kcb, P.nb - kc * P.kcb);
        for (int bl = 0; bl < nblk && ok;) {
          // Up to kG blocks per round when every token fits in the first 8
          // columns: their TMEM loads are all issued before one wait.
          const int g = nj <= 8 ? min(kG, nblk - bl) : 1;
          int tsi[kG];
          uint32_t phi[kG];
#pragma unroll
          for (int i = 0; i < kG; ++i) {
            tsi[i] = ts + i;
            phi[i] = tph;
            if (tsi[i] >= P.tb) {
              tsi[i] -= P.tb;
              phi[i] ^= 1;
            }
          }
#pragma unroll
          for (int i = 0; i < kG; ++i) {
            if (i < g && ok) ok = wait_bar(&B->tmem_full[tsi[i]], phi[i], B, P.err);
            if (i < g && ok) ok = wait_bar(&B->dw_full[tsi[i]], phi[i], B, P.err);
          }
          if (!ok) break;
          fence_after();
          if (nj <= 8) {
            uint32_t v[kG][NA][8];
#pragma unroll
            for (int i = 0; i < kG; ++i)
#pragma unroll
              for (int a = 0; a < NA; ++a)
                if (i < g) tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + tsi[i] * CPB + a * NT + j0, v[i][a]);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < kG; ++i) {
              if (i < g) {
                const int2* scb = sc + (bl + i) * NT + j0;
#pragma unroll
                for (int a = 0; a < NA; ++a) {
                  const float dw = dwr[tsi[i] * (NA * kM) + a * kM + 32 * q + lane];
#pragma unroll
                  for (int t = 0; t < 8; ++t) {
                    if (t < nj) {
                      const int2 s2 = scb[t];
                      const float isum = __fsub_rn(__int_as_float((int)v[i][a][t] + s2.y), kMagicF);
                      const float scale = __fmul_rn(dw, __int_as_float(s2.x));
                      acc[a][t] = __fadd_rn(acc[a][t], __fmul_rn(isum, scale));
                    }
                  }
                }
              }
            }
          } else {
            const int2* scb = sc + bl * NT + j0;
#pragma unroll
            for (int a = 0; a < NA; ++a) {
              const float dw = dwr[ts * (NA * kM) + a * kM + 32 * q + lane];
#pragma unroll
              for (int c8 = 0; c8 < TPW; c8 += 8) {
                if (c8 < nj) {
                  uint32_t v[8];
                  tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + ts * CPB + a * NT + j0 + c8, v);
                  tmem_wait_ld();
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    if (c8 + i < nj) {
                      const int2 s2 = scb[c8 + i];
                      const float isum = __fsub_rn(__int_as_float((int)v[i] + s2.y), kMagicF);
                      const float scale = __fmul_rn(dw, __int_as_float(s2.x));
                      acc[a][c8 + i] = __fadd_rn(acc[a][c8 + i], __fmul_rn(isum, scale));
                    }
                  }
                }
              }
            }
          }
          fence_before();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int i = 0; i < kG; ++i) {
              if (i < g) {
                mbar_arrive(&B->tmem_empty[tsi[i]]);
                mbar_arrive(&B->dw_empty[tsi[i]]);
              }
            }
          }
          ts += g;
          if (ts >= P.tb) {
            ts -= P.tb;
            tph ^= 1;
          }
          bl += g;
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&B->bs_empty[bsi]);
        if (++bsi == P.bs) {
          bsi = 0;
          bph ^= 1;
        }
      }
      if (!ok) break;
      // Unit outputs.
      if constexpr (MODE == kGateUp) {
        // act = gelu(gate) * up (ops.rs:99-114) for rows < I, then the down
        // product's Q8_0 re-quantisation (quant.rs:193-228): the warp's 32
        // lanes are the 32 elements of one act block.
        if (m0 + 32 * q < P.rows) {
          const int blk = (m0 + 32 * q) >> 5;
#pragma unroll
          for (int j = 0; j < TPW; ++j) {
            if (j < nj) {
              const float v = __fmul_rn(gelu_approx(acc[0][j]), acc[1][j]);
              float amax = fabsf(v);
              if (!(amax > 0.f)) amax = 0.f;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
              const float scale = __fdiv_rn(amax, 127.0f);
              const uint32_t d16 = f32_to_f16_trunc(scale);
              const float id = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
              float rq = round_half_away(__fmul_rn(v, id));
              if (rq != rq) rq = 0.f;
              rq = fminf(fmaxf(rq, -128.f), 127.f);
              const int qv = (int)rq;
              int qsum = qv;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
              const int pos = p0 + j0 + j;
              uint8_t* dst = reinterpret_cast<uint8_t*>(P.out_q) +
                             act_group_offset(false, blk, pos >> 3, 0, P.npad) + (lane >> 4) * 128 + (pos & 7) * 16 +
                             (lane & 15);
              *dst = (uint8_t)(int8_t)qv;
              if (lane == 0) {
                const int corr = P.down_q4 ? kMagicI - 8 * qsum : kMagicI;
                P.out_s[act_scale_index(blk, pos, P.npad)] = make_int2(__float_as_int(f16_bits_to_f32(d16)), corr);
              }
            }
          }
        }
      } else {
        if (row < P.rows) {
#pragma unroll
          for (int j = 0; j < TPW; ++j)
            if (j < nj) P.y[(size_t)(p0 + j0 + j) * P.rows + row] = acc[0][j];
        }
      }
    }
  }

  // Teardown: every role has left its loop (normally or on abort).
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

}  // namespace tc

// ---------------------------------------------------------------- host side

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D map over the gate/up weights viewed as 16-bit elements:
// {row_bytes/2, I rows, 2E parts} with a box of {8 blocks, box_rows rows, 1}.
bool make_gate_up_map(CUtensorMap* m, const uint8_t* w, int wtype, int H, int I, int E, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int bb = block_bytes(wtype);
  const cuuint64_t row_bytes = (cuuint64_t)(H / 32) * bb;
  cuuint64_t dims[3] = {row_bytes / 2, (cuuint64_t)I, (cuuint64_t)2 * E};
  cuuint64_t strides[2] = {row_bytes, row_bytes * I};
  cuuint32_t box[3] = {(cuuint32_t)(tc::kKC * bb / 2), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static std::atomic<int> n[kMaxDevices];
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && (v = n[dev].load(std::memory_order_relaxed)) > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return 148;
  if (dev >= 0 && dev < kMaxDevices) n[dev].store(v, std::memory_order_relaxed);
  return v;
}

constexpr int kSmemLimit = 227 * 1024;

struct Plan {
  int rs, as, bs, tb, raw_bytes, kcb;
  size_t smem;
};

Plan plan_for(int mode, int wtype, int NT, int nb, int rows_other, int row_bytes) {
  (void)rows_other;
  Plan p{};
  const int bb = block_bytes(wtype);
  const int na = mode == tc::kGateUp ? 2 : 1;
  const int slot = na * tc::kM * 32;
  p.kcb = mode == tc::kGateUp ? tc::kKC : nb;
  const int raw1 = mode == tc::kGateUp ? 2 * tc::kM * tc::kKC * bb : tc::kM * row_bytes;
  p.raw_bytes = (raw1 + 1023) & ~1023;
  p.tb = std::min(tc::kMaxRing, 512 / (na * NT));
  const int dw = p.tb * na * tc::kM * 4;
  const int bs_stage = p.kcb * NT * 40;
  // Prefer a deep raw (HBM) ring, then A-tile and B-stage depth.
  for (int rs = tc::kMaxRaw; rs >= 1; --rs)
    for (int bs = 4; bs >= 1; --bs)
      for (int as = 8; as >= 2; as /= 2) {
        const size_t total = 2048 + (size_t)rs * p.raw_bytes + (size_t)as * slot + dw + (size_t)bs * bs_stage;
        if (total <= (size_t)kSmemLimit) {
          p.rs = rs;
          p.bs = bs;
          p.as = as;
          // At least ~116 KB so that a single CTA owns the SM's TMEM.
          p.smem = std::max<size_t>(total, 116 * 1024);
          return p;
        }
      }
  p.smem = 0;
  return p;
}

template <int WQ4, int MODE, int NT>
cudaError_t launch_one(const CUtensorMap& map, const tc::Params& P, size_t smem, int grid, cudaStream_t s) {
  auto kern = tc::moe_gemm_tc_kernel<WQ4, MODE, NT>;
  static SmemOptIn cache;
  const cudaError_t st = ensure_smem(kern, smem, cache);
  if (st != cudaSuccess) return st;
  constexpr int threads = 32 * (tc::kEpiWarp0 + 4 * ((NT + 31) / 32));
  kern<<<grid, threads, smem, s>>>(map, P);
  return cudaPeekAtLastError();
}

}  // namespace

bool tc_map_available() { return encode_fn() != nullptr; }

bool tc_make_gate_up_map(CUtensorMap* m, const uint8_t* w, int wtype, int H, int I, int E, int box_rows) {
  return make_gate_up_map(m, w, wtype, H, I, E, box_rows);
}

int tc_num_sms() { return num_sms(); }

bool tc_supported(int wtype, int H, int I, int NT) {
  const int bbw = block_bytes(wtype);
  if (H % 256 != 0 || I % 32 != 0 || H % 32 != 0) return false;
  if (!encode_fn()) return false;
  const int down_row = (I / 32) * bbw;
  if (((size_t)32 * down_row) % 16 != 0) return false;
  if (plan_for(tc::kGateUp, wtype, NT, H / 32, 0, 0).smem == 0) return false;
  if (plan_for(tc::kDown, wtype, NT, I / 32, 0, down_row).smem == 0) return false;
  return true;
}

cudaError_t launch_gemm_tc(int mode, int wtype, int NT, const uint8_t* weights, int H, int I, int E, const int8_t* bq,
                           const int2* bsc, const int4* units, const int* n_units, int max_units, int npad,
                           int8_t* out_q, int2* out_s, float* y, int* err, cudaStream_t s) {
  tc::Params P{};
  const int bb = block_bytes(wtype);
  P.bq = bq;
  P.bsc = bsc;
  P.units = units;
  P.n_units = n_units;
  P.npad = npad;
  P.w_q4 = wtype == kQ4_0;
  P.err = err;
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  Plan pl;
  if (mode == tc::kGateUp) {
    P.nb = H / 32;
    P.rows = I;
    P.row_bytes = (H / 32) * bb;
    P.out_q = out_q;
    P.out_s = out_s;
    P.down_q4 = wtype == kQ4_0;
    if (!make_gate_up_map(&map, weights, wtype, H, I, E, tc::kM)) return cudaErrorInvalidValue;
    pl = plan_for(mode, wtype, NT, P.nb, 0, P.row_bytes);
  } else {
    P.nb = I / 32;
    P.rows = H;
    P.row_bytes = (I / 32) * bb;
    P.w_raw = weights;
    P.y = y;
    pl = plan_for(mode, wtype, NT, P.nb, 0, P.row_bytes);
  }
  if (pl.smem == 0) return cudaErrorInvalidValue;
  P.rs = pl.rs;
  P.as = pl.as;
  P.bs = pl.bs;
  P.tb = pl.tb;
  P.raw_bytes = pl.raw_bytes;
  P.kcb = pl.kcb;
  const int grid = std::max(1, std::min(num_sms(), max_units));
  const bool q4 = wtype == kQ4_0;
  if (mode == tc::kGateUp) {
    if (NT == 16) return q4 ? launch_one<1, tc::kGateUp, 16>(map, P, pl.smem, grid, s)
                            : launch_one<0, tc::kGateUp, 16>(map, P, pl.smem, grid, s);
    return q4 ? launch_one<1, tc::kGateUp, 64>(map, P, pl.smem, grid, s)
              : launch_one<0, tc::kGateUp, 64>(map, P, pl.smem, grid, s);
  }
  if (NT == 16) return q4 ? launch_one<1, tc::kDown, 16>(map, P, pl.smem, grid, s)
                          : launch_one<0, tc::kDown, 16>(map, P, pl.smem, grid, s);
  return q4 ? launch_one<1, tc::kDown, 64>(map, P, pl.smem, grid, s)
            : launch_one<0, tc::kDown, 64>(map, P, pl.smem, grid, s);
}

}  // namespace mrml
