// gemv.cu — grouped expert products for decode-size work (and prefill).
//
// When an expert sees only a few tokens, one tcgen05.mma per 32-element
// quant block keeps the tensor pipe busy ~160 cycles whatever the token
// count, which caps a Q4_0 layer well below the HBM rate.  This kernel keeps
// the same warp-specialised TMA pipeline as gemm_tc.cu:
//   warp 0       weight producer (TMA tensor-map tiles / 1-D bulk rows)
//   warp 1       activation producer (B tiles and scale records, bulk copies)
//   warps 2..5   compute, 128 weight rows x one unit of up to 8 positions.
//                For gate/up, warps 2-3 hold the 64 gate rows and warps 4-5
//                the matching up rows; at the end of a unit the up rows' sums
//                pass to the gate warps through shared memory, which apply
//                GeGLU and the Q8_0 quantisation of the down product's input.
// Two compute forms: MMA = 1, warp-level mma.sync m16n8k32 block dots (the
// automatic choice from a quarter of a (token, slot) pair per expert), and
// MMA = 0, dp4a with one weight row per thread (the smallest batches).
// The per-row f32 chain sum += (float)isum_b * (d_w * d_a) runs in block
// order, as in the reference (quant.rs:335-369 / 564-577), so the results
// are bit-identical to the tensor-core kernel and to the reference.
#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"

namespace mrml {
namespace gv {

using tc::GvBars;
using tc::kDown;
using tc::kGateUp;
using tc::kKC;
using tc::kM;
using tc::Params;
using tc::wait_bar;

// CTAs per SM of the warp-MMA gate/up kernel with one position group per
// unit (its launch bound: 5 leaves 64 registers per thread).
#ifndef MRML_GV_GATE_UP_CTAS
#define MRML_GV_GATE_UP_CTAS 5
#endif
constexpr int kGateUpCtas = MRML_GV_GATE_UP_CTAS;

// CTAs per SM of each form (its launch bound): the MMA gate/up product with
// one position group per unit kGateUpCtas; 16-position units on packed
// weights or Q8_0 rows 3 (their accumulators need the registers: at 4 the
// packed Q4_0 gate/up spilled and took 3.67 ms at config 4 against 3.26 ms at
// 3), on Q4_0 GGUF rows 4 (3.33 against 3.77 ms); the others 4.
__host__ __device__ constexpr int ctas_per_sm(bool mma, int mode, int ng, bool q4, bool packed) {
  return (mma && mode == kGateUp && ng == 1) ? kGateUpCtas : (ng == 2 && (packed || !q4) ? 3 : 4);
}

constexpr int kComp0 = 2;      // first compute warp
constexpr int kCompWarps = 4;  // 128 threads, one weight row each

// Integer dot of one weight block (8 words: Q4_0 nibbles or Q8_0 values in
// element order) with a token's 32 activation bytes, as the bits of the float
// 1.5*2^23 + isum: the correction word carries the magic (and, for Q4_0, the
// -8 * sum(q) nibble offset).  Two partial chains halve the dp4a depth.
template <int WQ4>
__device__ __forceinline__ int block_isum_bits(const uint32_t (&w)[8], const uint4& alo, const uint4& ahi, int corr) {
  int s0 = corr, s1 = 0;
  if constexpr (WQ4) {
    s0 = dp4a_us(w[0], alo.x, s0);
    s1 = dp4a_us(w[1], alo.y, s1);
    s0 = dp4a_us(w[2], alo.z, s0);
    s1 = dp4a_us(w[3], alo.w, s1);
    s0 = dp4a_us(w[4], ahi.x, s0);
    s1 = dp4a_us(w[5], ahi.y, s1);
    s0 = dp4a_us(w[6], ahi.z, s0);
    s1 = dp4a_us(w[7], ahi.w, s1);
  } else {
    s0 = dp4a_ss(w[0], alo.x, s0);
    s1 = dp4a_ss(w[1], alo.y, s1);
    s0 = dp4a_ss(w[2], alo.z, s0);
    s1 = dp4a_ss(w[3], alo.w, s1);
    s0 = dp4a_ss(w[4], ahi.x, s0);
    s1 = dp4a_ss(w[5], ahi.y, s1);
    s0 = dp4a_ss(w[6], ahi.z, s0);
    s1 = dp4a_ss(w[7], ahi.w, s1);
  }
  return s0 + s1;
}

// Raw block -> 8 words in element order: Q4_0 low nibbles (elements 0..15)
// then high nibbles (16..31); Q8_0 values as stored.
template <int WQ4>
__device__ __forceinline__ void block_words(const uint32_t* qs, uint32_t (&w)[8]) {
  if constexpr (WQ4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = qs[i] & 0x0f0f0f0fu;
      w[4 + i] = (qs[i] >> 4) & 0x0f0f0f0fu;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = qs[i];
  }
}

// One quant block of a weight row against the unit's tokens:
//   acc[t] += isum(t) * (d_w * d_a(t))
// in the reference's rounding order (scalar round-to-nearest operations; a
// packed f32x2 version of this sequence did not reproduce the scalar bits).
// btile: the block's 8-position activation group; rec: its group-major
// scale record ({d_a, correction} of the positions).
template <int WQ4, int TT>
__device__ __forceinline__ void block_tokens(const uint32_t (&w)[8], float dw, const uint8_t* btile, const uint8_t* rec,
                                             int nj, float (&acc)[TT]) {
  // Tokens in pairs: for even t the record holds {d(t), d(t+1), d(t),
  // d(t+1)} and {corr(t), corr(t+1), ...} as 16-byte groups, one load each.
#pragma unroll
  for (int t = 0; t < TT; t += 2) {
    if (t < nj) {
      const int4 dd = *reinterpret_cast<const int4*>(rec + 8 * t);
      const int2 cc = *reinterpret_cast<const int2*>(rec + 64 + 8 * t);
#pragma unroll
      for (int k = 0; k < 2 && t + k < TT; ++k) {
        if (k == 0 || t + 1 < nj) {
          const uint8_t* a = btile + (t + k) * 16;
          const uint4 alo = *reinterpret_cast<const uint4*>(a);
          const uint4 ahi = *reinterpret_cast<const uint4*>(a + 128);
          const float da = __int_as_float(k ? dd.y : dd.x);
          const float f =
              __fsub_rn(__int_as_float(block_isum_bits<WQ4>(w, alo, ahi, k ? cc.y : cc.x)), kMagicF);  // exact
          acc[t + k] = __fadd_rn(acc[t + k], __fmul_rn(f, __fmul_rn(dw, da)));
        }
      }
    }
  }
}

// ---------------------------------------------------- warp-level MMA path
// For units with several tokens, the integer block dots run on the tensor
// cores through mma.sync m16n8k32 (A = 16 weight rows x one 32-element
// quant block, B = the block's activations of the unit's 8 positions),
// which replaces 8 dp4a per (row, token, block) by one instruction per
// 16 rows x 8 tokens.  The accumulator is seeded with the same correction
// word as the dp4a chain (magic, and -8*sum(a) for Q4_0's unsigned
// nibbles), so D holds the bits of 1.5*2^23 + isum exactly, and the f32
// chain that follows is the reference's, element by element.
//
// Fragment layouts (PTX ISA, mma.m16n8k32 with 8-bit operands), lane =
// 4*g + t: a0/a2 = row g, elements 4t..4t+3 / 16+4t..; a1/a3 = row g+8;
// b0/b1 = position g, elements 4t.. / 16+4t..; d0,d1 = row g, positions
// 2t, 2t+1; d2,d3 = row g+8.
template <int WQ4>
__device__ __forceinline__ void mma_block(uint32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          const uint4& c) {
  if constexpr (WQ4)
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c.x), "r"(c.y), "r"(c.z), "r"(c.w));
  else
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c.x), "r"(c.y), "r"(c.z), "r"(c.w));
}

// A 32-bit word of shared memory at an address that is 4-byte aligned
// (ODD) or 2 bytes past a 4-byte boundary.
template <bool ALIGNED>
__device__ __forceinline__ uint32_t lds_word(const uint8_t* p) {
  if constexpr (ALIGNED) {
    return *reinterpret_cast<const uint32_t*>(p);
  } else {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - 2);
    return __funnelshift_r(q[0], q[1], 16);
  }
}

// Row fragment of one quant block for lane t: the low (elements 4t..) and
// high (16+4t..) words as unsigned nibbles (Q4_0) or signed bytes (Q8_0).
// A block's values start 2 bytes after its (2-byte aligned) start; blocks
// with an odd index within a 4-byte aligned row have them 4-byte aligned.
template <int WQ4, bool ODD>
__device__ __forceinline__ void block_frag(const uint8_t* blk, int t, uint32_t& lo, uint32_t& hi) {
  if constexpr (WQ4) {
    const uint32_t w = lds_word<ODD>(blk + 2 + 4 * t);
    lo = w & 0x0f0f0f0fu;
    hi = (w >> 4) & 0x0f0f0f0fu;
  } else {
    lo = lds_word<ODD>(blk + 2 + 4 * t);
    hi = lds_word<ODD>(blk + 18 + 4 * t);
  }
}

// Packed f32x2 arithmetic (sm_100): two independent IEEE round-to-nearest
// operations per instruction, lane for lane the scalar results.  Measured
// on B200 with CUDA 12.9: a packed multiply whose result feeds a packed add
// is contracted into a fused multiply-add despite the .rn modifiers, which
// changes the rounding; a packed multiply followed by scalar add.rn is not.
// So the chain's additions are packed fused multiply-adds acc + p * one,
// with `one` = 1.0 passed in at run time: p * 1.0 is exact, so the single
// rounding is that of the addition, and the compiler cannot fold the product
// that feeds p into the FMA, as it would for a literal 1.0 or a plain add.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// acc pair += p (one = {1.0, 1.0}, opaque): two round-to-nearest additions.
__device__ __forceinline__ void f2_acc(float& a0, float& a1, uint64_t p, uint64_t one) {
  f2_unpack(f2_fma(p, one, f2_pack(a0, a1)), a0, a1);
}

// Fragment loaders of the MMA path: lane (g, t)'s A fragment of one 16-row
// tile and one quant block (a0/a2 = row g, elements 4t.. / 16+4t..; a1/a3 =
// row g+8) and the two rows' scales {d_w(g), d_w(g+8)} as an f32 pair.
//
// Raw GGUF rows staged in shared memory: row g of the tile at `ra`, the block
// `boff` bytes into the row; blocks of odd index in a 4-byte aligned row have
// their values 4-byte aligned (ODD), even ones 2 bytes past.
template <int WQ4, bool ODD>
struct RawFrag {
  const uint8_t* row0;
  int pitch, boff;
  __device__ __forceinline__ void operator()(int i, int g, int t, uint32_t (&a)[4], uint64_t& dw) const {
    const uint8_t* ra = row0 + (16 * i + g) * pitch + boff;
    const uint8_t* rb = ra + 8 * pitch;
    block_frag<WQ4, ODD>(ra, t, a[0], a[2]);
    block_frag<WQ4, ODD>(rb, t, a[1], a[3]);
    dw = f2_pack(f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ra)),
                 f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rb)));
  }
};

// Packed weights (mrml_moe_prepare_weights): one record per (16-row tile,
// block) in MMA fragment order, 16 * block_bytes long.  Q4_0: lane l = 4g+t
// owns bytes [8l, 8l+8) = the raw nibble bytes [4t, 4t+4) of rows g and g+8;
// Q8_0: bytes [16l, 16l+16) = rows g, g+8 values [4t, 4t+4), then rows g,
// g+8 values [16+4t, 16+4t+4).  The 16 f16 scales follow the values as
// pairs {d(g), d(g+8)}.  `rec` is tile 0's record; tile i's is rstep bytes on.
template <int WQ4>
struct PackedFrag {
  const uint8_t* rec;
  int rstep;
  __device__ __forceinline__ void operator()(int i, int g, int t, uint32_t (&a)[4], uint64_t& dw) const {
    const uint8_t* r = rec + i * rstep;
    const int lane = 4 * g + t;
    uint32_t s;
    if constexpr (WQ4) {
      const uint2 w = *reinterpret_cast<const uint2*>(r + 8 * lane);
      a[0] = w.x & 0x0f0f0f0fu;
      a[2] = (w.x >> 4) & 0x0f0f0f0fu;
      a[1] = w.y & 0x0f0f0f0fu;
      a[3] = (w.y >> 4) & 0x0f0f0f0fu;
      s = *reinterpret_cast<const uint32_t*>(r + 256 + 4 * g);
    } else {
      const uint4 w = *reinterpret_cast<const uint4*>(r + 16 * lane);
      a[0] = w.x;
      a[1] = w.y;
      a[2] = w.z;
      a[3] = w.w;
      s = *reinterpret_cast<const uint32_t*>(r + 512 + 4 * g);
    }
    dw = f2_pack(f16_bits_to_f32(s & 0xffffu), f16_bits_to_f32(s >> 16));
  }
};

// One quant block for the warp's two 16-row tiles (rows 16i+g, 16i+g+8) and
// the unit's NG position groups of 8:
//   acc[8q + 4i + 2h + k] += isum * (d_w(row 16i + 8h + g) * d_a(8q + 2t + k))
// grp: group 0's activations of the block, the next group gstride bytes on;
// rec: group 0's group-major scale record (rstride bytes to the next), from
// which lane t takes the d_a pair of columns 2t, 2t+1 and the accumulator
// seeds with one load each.  The chain runs on packed column pairs of one
// row, the MMA's own accumulator register pairs (d0, d1) and (d2, d3): the
// pair's d_w is the row's scale twice and d_a the record's pair, so no
// accumulator is moved between registers.  A row fragment is loaded and
// unpacked once for all NG groups.
template <int WQ4, int NG, class Frag>
__device__ __forceinline__ void mma_block_rows2(const Frag& frag, const uint8_t* grp, int gstride, const uint8_t* rec,
                                                int rstride, uint64_t one, int g, int t, float (&acc)[8 * NG]) {
  uint32_t b0[NG], b1[NG];
  uint4 seed[NG];
  uint64_t da[NG];
#pragma unroll
  for (int q = 0; q < NG; ++q) {
    b0[q] = *reinterpret_cast<const uint32_t*>(grp + q * gstride + g * 16 + 4 * t);
    b1[q] = *reinterpret_cast<const uint32_t*>(grp + q * gstride + 128 + g * 16 + 4 * t);
    seed[q] = *reinterpret_cast<const uint4*>(rec + q * rstride + 64 + 16 * t);
    da[q] = *reinterpret_cast<const uint64_t*>(rec + q * rstride + 16 * t);
  }
  const uint64_t magic = f2_pack(kMagicF, kMagicF);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint32_t a[4];
    uint64_t dw;
    frag(i, g, t, a, dw);
    float dwg, dwg8;
    f2_unpack(dw, dwg, dwg8);
    const uint64_t dw0 = f2_pack(dwg, dwg), dw1 = f2_pack(dwg8, dwg8);
#pragma unroll
    for (int q = 0; q < NG; ++q) {
      uint32_t d[4];
      mma_block<WQ4>(d, a, b0[q], b1[q], seed[q]);
      const uint64_t f0 = f2_sub(f2_pack(__uint_as_float(d[0]), __uint_as_float(d[1])), magic);  // exact
      const uint64_t f1 = f2_sub(f2_pack(__uint_as_float(d[2]), __uint_as_float(d[3])), magic);
      float* aq = acc + 8 * q + 4 * i;
      f2_acc(aq[0], aq[1], f2_mul(f0, f2_mul(dw0, da[q])), one);
      f2_acc(aq[2], aq[3], f2_mul(f1, f2_mul(dw1, da[q])), one);
    }
  }
}

// The same block for a down unit of at most 4 tokens.  The warp's two 16-row MMAs
// see the positions in order (rows 0-15) and rotated by 4 (rows 16-31), so
// the valid columns of the first land in lanes t = 0, 1 and those of the
// second in lanes t = 2, 3; each lane runs the f32 chain for one of the two
// (half the chain work of mma_block_rows2, which computes all 8 columns).
// acc[2h + k]: tile row 16*(t >> 1) + 8h + g, position 2*(t & 1) + k; the
// d_a pairs and seeds come from positions 2*(t & 1) and 2*(t & 1) + 1.
template <int WQ4, class Frag>
__device__ __forceinline__ void mma_block_rows2_half(const Frag& frag, const uint8_t* grp, const uint8_t* rec,
                                                     uint64_t one, int g, int t, float (&acc)[4]) {
  const int th = t & 1;
  const uint4 seed = *reinterpret_cast<const uint4*>(rec + 64 + 16 * th);
  const uint32_t b0 = *reinterpret_cast<const uint32_t*>(grp + g * 16 + 4 * t);
  const uint32_t b1 = *reinterpret_cast<const uint32_t*>(grp + 128 + g * 16 + 4 * t);
  const uint32_t r0 = *reinterpret_cast<const uint32_t*>(grp + (g ^ 4) * 16 + 4 * t);
  const uint32_t r1 = *reinterpret_cast<const uint32_t*>(grp + 128 + (g ^ 4) * 16 + 4 * t);
  uint32_t a[4], d0[4], d1[4];
  uint64_t dw0, dw1;
  frag(0, g, t, a, dw0);
  mma_block<WQ4>(d0, a, b0, b1, seed);
  frag(1, g, t, a, dw1);
  mma_block<WQ4>(d1, a, r0, r1, seed);
  const bool hi = t >= 2;
  uint32_t d[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) d[j] = hi ? d1[j] : d0[j];
  float dwg, dwg8;
  f2_unpack(hi ? dw1 : dw0, dwg, dwg8);
  const uint64_t da = *reinterpret_cast<const uint64_t*>(rec + 16 * th);
  const uint64_t magic = f2_pack(kMagicF, kMagicF);
  const uint64_t f0 = f2_sub(f2_pack(__uint_as_float(d[0]), __uint_as_float(d[1])), magic);  // exact
  const uint64_t f1 = f2_sub(f2_pack(__uint_as_float(d[2]), __uint_as_float(d[3])), magic);
  f2_acc(acc[0], acc[1], f2_mul(f0, f2_mul(f2_pack(dwg, dwg), da)), one);
  f2_acc(acc[2], acc[3], f2_mul(f1, f2_mul(f2_pack(dwg8, dwg8), da)), one);
}

// The K chunks of one unit on the dp4a path, for compute thread row `c`:
// NJ accumulators, of which the first nj hold tokens (NJ = 1 for the units
// of a single token, the common case of the smallest batches, so that
// their blocks carry no predicated work for absent tokens).  Ring indices
// and phases advance as the caller's.  Returns false when a wait gave up.
// Row `r` (0..15) of a packed record (PackedFrag's layout) as the raw
// block's values in element order's storage words and its f16 scale.
template <int WQ4>
__device__ __forceinline__ void packed_row(const uint8_t* rec, int r, uint32_t& d16,
                                           uint32_t (&qs)[WQ4 ? 4 : 8]) {
  const int g = r & 7, h = r >> 3;
  if constexpr (WQ4) {
#pragma unroll
    for (int t = 0; t < 4; ++t) qs[t] = *reinterpret_cast<const uint32_t*>(rec + 8 * (4 * g + t) + 4 * h);
    d16 = *reinterpret_cast<const uint16_t*>(rec + 256 + 4 * g + 2 * h);
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      qs[t] = *reinterpret_cast<const uint32_t*>(rec + 16 * (4 * g + t) + 4 * h);
      qs[4 + t] = *reinterpret_cast<const uint32_t*>(rec + 16 * (4 * g + t) + 8 + 4 * h);
    }
    d16 = *reinterpret_cast<const uint16_t*>(rec + 512 + 4 * g + 2 * h);
  }
}

template <int WQ4, int MODE, int NJ, int PK>
__device__ __forceinline__ bool dp4a_chunks(const Params& P, GvBars* B, const uint8_t* raw, const uint8_t* bsb,
                                            int bs_stage, int nkc, int c, int nj, int& rs, int& bsi, uint32_t& rph,
                                            uint32_t& bph, float (&acc)[NJ]) {
  constexpr int BB = WQ4 ? 18 : 34;
  constexpr int GB = 256;
  constexpr int RB = 16 * BB;  // packed record bytes
  const int lane = threadIdx.x & 31;
  for (int kc = 0; kc < nkc; ++kc) {
    if (!wait_bar(&B->raw_full[rs], rph, B, P.err)) return false;
    if (!wait_bar(&B->bs_full[bsi], bph, B, P.err)) return false;
    const uint8_t* src = raw + rs * P.raw_bytes;
    const uint8_t* bt = bsb + bsi * bs_stage;
    const uint8_t* sc = bt + P.kcb * GB;  // the blocks' group-major scale records
    if constexpr (PK) {
      // Stage: gate/up [part][tile 4][block kKC][RB] (thread c = part * 64 +
      // 16 * tile + row); down [tile 8][block kcb][RB].
      const int nbs = MODE == kGateUp ? kKC : P.kcb;
      const uint8_t* tile = src + (size_t)(c >> 4) * nbs * RB;
      for (int b = 0; b < nbs; ++b) {
        uint32_t d16, q[WQ4 ? 4 : 8], w[8];
        packed_row<WQ4>(tile + b * RB, c & 15, d16, q);
        block_words<WQ4>(q, w);
        block_tokens<WQ4, NJ>(w, f16_bits_to_f32(d16), bt + b * GB, sc + b * kActScaleBytes, nj, acc);
      }
    } else if constexpr (MODE == kGateUp) {
      const uint8_t* row = src + c * (kKC * BB);  // gate rows 0..63, then up rows
#define MRML_GV_BLOCK(BL)                                                                     \
  {                                                                                           \
    uint32_t d16, q[BB == 18 ? 4 : 8], w[8];                                                  \
    tc::chunk_block<BB, BL>(row, d16, q);                                                     \
    block_words<WQ4>(q, w);                                                                   \
    block_tokens<WQ4, NJ>(w, f16_bits_to_f32(d16), bt + (BL) * GB, sc + (BL) * kActScaleBytes, nj, acc); \
  }
      MRML_GV_BLOCK(0) MRML_GV_BLOCK(1) MRML_GV_BLOCK(2) MRML_GV_BLOCK(3)
      MRML_GV_BLOCK(4) MRML_GV_BLOCK(5) MRML_GV_BLOCK(6) MRML_GV_BLOCK(7)
#undef MRML_GV_BLOCK
    } else {
      const uint8_t* row = src + (size_t)c * P.row_bytes;
      for (int b = 0; b < P.nb; ++b) {
        uint32_t w[8];
        uint32_t d16;
        if constexpr (WQ4) {
          const Q4Block q = load_q4_block(row + b * 18);
          d16 = q.d16;
          block_words<1>(q.qs, w);
        } else {
          const Q8Block q = load_q8_block(row + b * 34);
          d16 = q.d16;
          block_words<0>(q.qs, w);
        }
        block_tokens<WQ4, NJ>(w, f16_bits_to_f32(d16), bt + b * GB, sc + b * kActScaleBytes, nj, acc);
      }
    }
    __syncwarp();
    if (lane == 0) {
      tc::mbar_arrive(&B->raw_empty[rs]);
      tc::mbar_arrive(&B->bs_empty[bsi]);
    }
    if (++rs == P.rs) {
      rs = 0;
      rph ^= 1;
    }
    if (++bsi == P.bs) {
      bsi = 0;
      bph ^= 1;
    }
  }
  return true;
}

// Unit: NG groups of kGvTokens (8) positions and 128 weight rows: for
// gate/up, gate rows m0..m0+63 and the same up rows; for down, rows
// m0..m0+127.  NG = 2 (the MMA form only) when experts see about 12 tokens
// or more: a weight stage then serves 16 positions, each row fragment is
// unpacked once for two MMAs, and the weights stream half as often.
// Activations use the group-major layout (common.cuh): a B stage holds, for
// each of the unit's groups, the chunk's blocks (256 bytes each, contiguous),
// then each group's scale records.
//
// PK = 1: the weights are in the packed layout of mrml_moe_prepare_weights
// (PackedFrag's records; per unit and K chunk contiguous), streamed with 1-D
// bulk copies: gate/up [E][part][64-row group][K chunk][tile 4][block
// kKC][record], down [E][128-row group][K chunk][tile 8][block
// down_chunk_blocks][record].
template <int WQ4, int MODE, int MMA, int NG, int PK>
__global__ void __launch_bounds__(32 * (kComp0 + kCompWarps),
                                  ctas_per_sm(MMA, MODE, NG, WQ4, PK))
    moe_gemv_kernel(const __grid_constant__ CUtensorMap tmap, const Params P) {
  static_assert(NG == 1 || (NG == 2 && MMA), "two position groups per unit on the MMA form only");
  constexpr int BB = WQ4 ? 18 : 34;
  constexpr int RB = 16 * BB;  // packed record bytes
  constexpr int TT = kGvTokens;
  constexpr int NP = TT * NG;  // positions per unit
  constexpr int RG = kGvRowsGateUp;  // row pairs per unit
  constexpr int GB = 256;            // bytes of one block's activation group
  constexpr int SB = kActScaleBytes;  // bytes of one block's scale record

  // 128-byte alignment is what the (unswizzled) tensor copies need; the
  // barrier block takes the first kGvBarBytes.
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  GvBars* B = reinterpret_cast<GvBars*>(smem);
  uint8_t* raw = smem + tc::kGvBarBytes;
  uint8_t* bsb = raw + P.rs * P.raw_bytes;
  const int bs_stage = P.kcb * NG * (GB + SB);
  float* xch = reinterpret_cast<float*>(bsb + P.bs * bs_stage);  // [NP][RG] up-row sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.rs; ++i) {
      mbar_init(&B->raw_full[i], 1);
      mbar_init(&B->raw_empty[i], kCompWarps);
    }
    for (int i = 0; i < P.bs; ++i) {
      mbar_init(&B->bs_full[i], 1);
      mbar_init(&B->bs_empty[i], kCompWarps);
    }
    mbar_init(&B->xch_full, kCompWarps / 2);
    mbar_init(&B->xch_empty, kCompWarps / 2);
    B->abort = 0;
    fence_barrier_init();
  }
  // Programmatic dependent launch: the work units and the weights were
  // complete before this grid started (the kernel before it waits for the
  // dispatch before triggering this launch, or is the dispatch kernel and
  // then does not trigger early; weights are never written),
  // so the weight producer streams right away; only the activation producer
  // waits for the previous kernel (whose output it reads), and the compute
  // warps consume nothing that has not passed through it.
  pdl_trigger();
  __syncthreads();
  const int n_units = *P.n_units;
  const int nkc = MODE == kGateUp ? P.nb / kKC : P.nb / P.kcb;

  if (warp == 0) {
    // ----------------------------------------------------- weight producer
    if (lane == 0) {
      int rs = 0;
      uint32_t rph = 0;
      for (int u = blockIdx.x; u < n_units && !tc::aborted(B); u += gridDim.x) {
        const int4 U = P.units[u];
        const int e = U.x, m0 = U.w;
        for (int kc = 0; kc < nkc; ++kc) {
          if (!wait_bar(&B->raw_empty[rs], rph ^ 1, B, P.err)) break;
          uint8_t* dst = raw + rs * P.raw_bytes;
          if constexpr (PK && MODE == kGateUp) {
            // gate part, then up part: 4 tiles x kKC blocks each
            const uint32_t part = 4 * kKC * RB;
            const int ng = P.rows / RG, nc = P.nb / kKC;
            mbar_arrive_expect_tx(&B->raw_full[rs], 2 * part);
            const uint8_t* gsrc = P.w_raw + ((((size_t)e * 2) * ng + m0 / RG) * nc + kc) * part;
            bulk_g2s(dst, gsrc, part, &B->raw_full[rs]);
            bulk_g2s(dst + part, gsrc + (size_t)ng * nc * part, part, &B->raw_full[rs]);
          } else if constexpr (PK) {
            // down: the unit's K chunk kc, 8 tiles x kcb blocks, one run
            const uint32_t bytes = (uint32_t)(8 * P.kcb * RB);
            mbar_arrive_expect_tx(&B->raw_full[rs], bytes);
            bulk_g2s(dst, P.w_raw + (((size_t)e * (P.rows / 128) + m0 / 128) * nkc + kc) * bytes, bytes,
                     &B->raw_full[rs]);
          } else if constexpr (MODE == kGateUp) {
            mbar_arrive_expect_tx(&B->raw_full[rs], 2 * RG * kKC * BB);
            const int c0 = kc * kKC * BB / 2;
            tc::tma_load_3d(dst, &tmap, c0, m0, 2 * e, &B->raw_full[rs]);
            tc::tma_load_3d(dst + RG * kKC * BB, &tmap, c0, m0, 2 * e + 1, &B->raw_full[rs]);
          } else {
            const int nrows = min(2 * RG, P.rows - m0);
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
  } else if (warp == 1) {
    // ------------------------------------------------- activation producer
    if (lane == 0) {
      pdl_wait();  // in every CTA, so the grid completes after its predecessor
      int bsi = 0;
      uint32_t bph = 0;
      for (int u = blockIdx.x; u < n_units && !tc::aborted(B); u += gridDim.x) {
        const int p0 = P.units[u].y;
        for (int kc = 0; kc < nkc; ++kc) {
          if (!wait_bar(&B->bs_empty[bsi], bph ^ 1, B, P.err)) break;
          uint8_t* bdst = bsb + bsi * bs_stage;
          const int b0 = kc * P.kcb;
          const int nblk = min(P.kcb, P.nb - b0);
          mbar_arrive_expect_tx(&B->bs_full[bsi], (uint32_t)(nblk * NG * (GB + SB)));
          // Group-major layout: a group's blocks b0 .. b0+nblk-1 are
          // contiguous, for the activations and for their scale records.
#pragma unroll
          for (int q = 0; q < NG; ++q) {
            const int g = (p0 >> 3) + q;
            bulk_g2s(bdst + q * P.kcb * GB, P.bq + act_group_offset(true, b0, g, P.nb, P.npad), nblk * GB,
                     &B->bs_full[bsi]);
            bulk_g2s(bdst + NG * P.kcb * GB + q * P.kcb * SB,
                     reinterpret_cast<const uint8_t*>(P.bsc) + act_scale_offset_gm(b0, 8 * g, P.nb), nblk * SB,
                     &B->bs_full[bsi]);
          }
          if (++bsi == P.bs) {
            bsi = 0;
            bph ^= 1;
          }
        }
      }
    }
  } else if constexpr (MMA) {
    // -------------------------------------------------- compute (mma.sync)
    // Compute warp cw owns tile rows 32cw .. 32cw+31 (gate/up: warps 0-1 the
    // gate rows, 2-3 the same up rows, lane for lane).
    const int cw = warp - kComp0;
    const int g = lane >> 2, t = lane & 3;
    const bool up_warp = MODE == kGateUp && cw >= kCompWarps / 2;
    const uint64_t one = f2_pack(P.one, P.one);
    int rs = 0, bsi = 0;
    uint32_t rph = 0, bph = 0, xph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok && !tc::aborted(B); u += gridDim.x) {
      const int4 U = P.units[u];
      const int p0 = U.y, nvalid = U.z, m0 = U.w;
      const int nj = min(NP, nvalid);
      float acc[8 * NG];
#pragma unroll
      for (int j = 0; j < 8 * NG; ++j) acc[j] = 0.f;
      // Q4_0 down units of at most 4 tokens run the half-chain form.  (For
      // gate/up it measured slower: a second unrolled chunk body in a kernel
      // held to 64 registers; for Q8_0 its registers spill.)
      // Down units of at most 4 positions run the half-chain form (Q4_0 rows
      // and packed weights).  For gate/up it measured slower (a second
      // unrolled chunk body; on GGUF rows held to 64 registers, on packed
      // weights 84.6 against 68.1 us at config 2, T = 64); for Q8_0 GGUF down
      // rows its registers spill.
      const bool half = MODE == kDown && (WQ4 || PK) && NG == 1 && nj <= 4;  // warp-uniform
      float(&acch)[4] = *reinterpret_cast<float(*)[4]>(&acc[0]);  // the half layout's sums
      for (int kc = 0; kc < nkc && ok; ++kc) {
        if (!(ok = wait_bar(&B->raw_full[rs], rph, B, P.err))) break;
        if (!(ok = wait_bar(&B->bs_full[bsi], bph, B, P.err))) break;
        const uint8_t* src = raw + rs * P.raw_bytes;
        const uint8_t* bt = bsb + bsi * bs_stage;
        const uint8_t* sc = bt + NG * P.kcb * GB;  // the blocks' group-major scale records
        const int gs = P.kcb * GB, ss = P.kcb * SB;  // strides between the unit's groups
        if constexpr (PK && MODE == kGateUp) {
          // warp cw: part cw / 2, tiles 2 (cw & 1) and 2 (cw & 1) + 1
          const uint8_t* t0 = src + (size_t)((cw >> 1) * 4 + 2 * (cw & 1)) * kKC * RB;
#pragma unroll
          for (int bl = 0; bl < kKC; ++bl)
            mma_block_rows2<WQ4, NG>(PackedFrag<WQ4>{t0 + bl * RB, kKC * RB}, bt + bl * GB, gs, sc + bl * SB, ss, one,
                                     g, t, acc);
        } else if constexpr (PK) {
          // down: this stage's K chunk of kcb blocks; warp cw's tiles 2cw, 2cw + 1
          const uint8_t* t0 = src + (size_t)(2 * cw) * P.kcb * RB;
          if (NG == 1 && half) {
#pragma unroll 2
            for (int b = 0; b < P.kcb; ++b)
              mma_block_rows2_half<WQ4>(PackedFrag<WQ4>{t0 + b * RB, P.kcb * RB}, bt + b * GB, sc + b * SB, one, g,
                                        t, acch);
          } else {
#pragma unroll 2
            for (int b = 0; b < P.kcb; ++b)
              mma_block_rows2<WQ4, NG>(PackedFrag<WQ4>{t0 + b * RB, P.kcb * RB}, bt + b * GB, gs, sc + b * SB, ss,
                                       one, g, t, acc);
          }
        } else if constexpr (MODE == kGateUp) {
          const uint8_t* row0 = src + 32 * cw * (kKC * BB);
#pragma unroll
          for (int bl = 0; bl < kKC; bl += 2) {
            mma_block_rows2<WQ4, NG>(RawFrag<WQ4, false>{row0, kKC * BB, bl * BB}, bt + bl * GB, gs, sc + bl * SB,
                                     ss, one, g, t, acc);
            mma_block_rows2<WQ4, NG>(RawFrag<WQ4, true>{row0, kKC * BB, (bl + 1) * BB}, bt + (bl + 1) * GB, gs,
                                     sc + (bl + 1) * SB, ss, one, g, t, acc);
          }
        } else {
          const uint8_t* row0 = src + (size_t)(32 * cw) * P.row_bytes;
          if (WQ4 && NG == 1 && half) {
#pragma unroll 1
            for (int b = 0; b < P.nb; b += 2) {
              mma_block_rows2_half<WQ4>(RawFrag<WQ4, false>{row0, P.row_bytes, b * BB}, bt + b * GB, sc + b * SB, one,
                                        g, t, acch);
              mma_block_rows2_half<WQ4>(RawFrag<WQ4, true>{row0, P.row_bytes, (b + 1) * BB}, bt + (b + 1) * GB,
                                        sc + (b + 1) * SB, one, g, t, acch);
            }
          } else {
#pragma unroll 1
            for (int b = 0; b < P.nb; b += 2) {
              mma_block_rows2<WQ4, NG>(RawFrag<WQ4, false>{row0, P.row_bytes, b * BB}, bt + b * GB, gs, sc + b * SB,
                                       ss, one, g, t, acc);
              mma_block_rows2<WQ4, NG>(RawFrag<WQ4, true>{row0, P.row_bytes, (b + 1) * BB}, bt + (b + 1) * GB, gs,
                                       sc + (b + 1) * SB, ss, one, g, t, acc);
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&B->raw_empty[rs]);
          tc::mbar_arrive(&B->bs_empty[bsi]);
        }
        if (++rs == P.rs) {
          rs = 0;
          rph ^= 1;
        }
        if (++bsi == P.bs) {
          bsi = 0;
          bph ^= 1;
        }
      }
      if (!ok) break;
      if (half) {
        // Back to the 8-position layout: lane (g, t < 2) keeps its rows
        // 0-15 and takes rows 16-31 of the same positions from lane t ^ 2;
        // lanes t >= 2 hold positions 4..7, absent in these units.
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float other = __shfl_xor_sync(0xffffffffu, acch[j], 2);
          if (t < 2) acc[4 + j] = other;
        }
      }
      // acc[8q + 4i + 2h + k]: tile row 32cw + 16i + 8h + g, position
      // p0 + 8q + 2t + k.
      if constexpr (MODE == kGateUp) {
        float* xw = xch + (cw & 1) * 8 * NG * 32;  // [8 NG][32 lanes] per gate/up warp pair
        if (up_warp) {
          if (!(ok = wait_bar(&B->xch_empty, xph ^ 1, B, P.err))) break;
#pragma unroll
          for (int j = 0; j < 8 * NG; ++j) xw[j * 32 + lane] = acc[j];
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&B->xch_full);
          xph ^= 1;
          continue;
        }
        if (!(ok = wait_bar(&B->xch_full, xph, B, P.err))) break;
        float upv[8 * NG];
#pragma unroll
        for (int j = 0; j < 8 * NG; ++j) upv[j] = xw[j * 32 + lane];
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&B->xch_empty);
        xph ^= 1;
        // act = gelu(gate) * up (ops.rs:99-114) and the down product's Q8_0
        // re-quantisation (quant.rs:193-228).  The warp's 32 rows are one act
        // block; the 8 lanes with the same t hold its 32 values for
        // positions 2t and 2t+1.
        const int rbase = m0 + 32 * cw;
        if (rbase < P.rows && NG == 1 && nj <= 4) {
          // Units of at most 4 positions: lanes t < 2 hold them, so each
          // lane pair (t, t ^ 2) splits the work — lane t keeps rows 0-15
          // of positions 2(t & 1) + k, lane t ^ 2 takes rows 16-31 — and a
          // lane evaluates 4 GeGLUs instead of 8.  Maxima and sums then
          // also reduce across the pair; both are order-independent, so the
          // results are those of the 8-position form.
          const int blk = rbase >> 5, th = t & 1, ih = t >> 1;
          float a4[4], u4[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float ra = __shfl_xor_sync(0xffffffffu, acc[4 + j], 2);
            const float ru = __shfl_xor_sync(0xffffffffu, upv[4 + j], 2);
            a4[j] = ih ? ra : acc[j];  // a4[2h + k]: row 16 ih + 8h + g, position 2 th + k
            u4[j] = ih ? ru : upv[j];
          }
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int pj = 2 * th + k;
            float v[2];
            float amax = 0.f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              v[h] = __fmul_rn(gelu_approx(a4[2 * h + k]), u4[2 * h + k]);
              float a = fabsf(v[h]);
              if (!(a > 0.f)) a = 0.f;
              amax = fmaxf(amax, a);
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float scale = __fdiv_rn(amax, 127.0f);
            const uint32_t d16 = f32_to_f16_trunc(scale);
            const float id = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
            int qv[2], qsum = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float rq = round_half_away(__fmul_rn(v[h], id));
              if (rq != rq) rq = 0.f;
              rq = fminf(fmaxf(rq, -128.f), 127.f);
              qv[h] = (int)rq;
              qsum += qv[h];
            }
            qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
            if (pj < nj) {
              const int pos = p0 + pj;
              uint8_t* dst = reinterpret_cast<uint8_t*>(P.out_q) + act_group_offset(true, blk, pos >> 3, P.out_nb, P.npad) +
                             (pos & 7) * 16;
#pragma unroll
              for (int h = 0; h < 2; ++h) {  // element 16 ih + 8h + g of the block
                const int e = 16 * ih + 8 * h + g;
                dst[(e >> 4) * 128 + (e & 15)] = (uint8_t)(int8_t)qv[h];
              }
              if (g == 0 && ih == 0) {
                const int corr = P.down_q4 ? kMagicI - 8 * qsum : kMagicI;
                store_act_scale_gm(P.out_s, blk, pos, P.out_nb, f16_bits_to_f32(d16), corr);
              }
            }
          }
        } else if (rbase < P.rows) {
          const int blk = rbase >> 5;
#pragma unroll
          for (int kk = 0; kk < 2 * NG; ++kk) {
            const int k = kk & 1, o8 = 8 * (kk >> 1);  // position 2t + k of group kk / 2
            const int pj = o8 + 2 * t + k;
            float v[4];
            float amax = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              v[q] = __fmul_rn(gelu_approx(acc[o8 + 2 * q + k]), upv[o8 + 2 * q + k]);
              float a = fabsf(v[q]);
              if (!(a > 0.f)) a = 0.f;
              amax = fmaxf(amax, a);
            }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float scale = __fdiv_rn(amax, 127.0f);
            const uint32_t d16 = f32_to_f16_trunc(scale);
            const float id = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
            int qv[4], qsum = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float rq = round_half_away(__fmul_rn(v[q], id));
              if (rq != rq) rq = 0.f;
              rq = fminf(fmaxf(rq, -128.f), 127.f);
              qv[q] = (int)rq;
              qsum += qv[q];
            }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
            if (pj < nj) {
              const int pos = p0 + pj;
              uint8_t* dst = reinterpret_cast<uint8_t*>(P.out_q) + act_group_offset(true, blk, pos >> 3, P.out_nb, P.npad) +
                             (pos & 7) * 16;
#pragma unroll
              for (int q = 0; q < 4; ++q) {  // element 16i + 8h + g of the block, q = 2i + h
                const int e = 8 * q + g;
                dst[(e >> 4) * 128 + (e & 15)] = (uint8_t)(int8_t)qv[q];
              }
              if (g == 0) {
                const int corr = P.down_q4 ? kMagicI - 8 * qsum : kMagicI;
                store_act_scale_gm(P.out_s, blk, pos, P.out_nb, f16_bits_to_f32(d16), corr);
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8 * NG; ++j) {
          const int row = m0 + 32 * cw + 8 * ((j & 7) >> 1) + g;  // 16i + 8h = 8 * (2i + h)
          const int pj = 8 * (j >> 3) + 2 * t + (j & 1);
          if (row < P.rows && pj < nj) P.y[(size_t)(p0 + pj) * P.rows + row] = acc[j];
        }
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    const int c = threadIdx.x - 32 * kComp0;  // raw-tile row of this thread
    const bool up_row = MODE == kGateUp && c >= RG;
    int rs = 0, bsi = 0;
    uint32_t rph = 0, bph = 0, xph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok && !tc::aborted(B); u += gridDim.x) {
      const int4 U = P.units[u];
      const int p0 = U.y, nvalid = U.z, m0 = U.w;
      const int nj = min(TT, nvalid);
      float acc[TT];
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[t] = 0.f;
      if (nj == 1) {
        float acc1[1] = {0.f};
        ok = dp4a_chunks<WQ4, MODE, 1, PK>(P, B, raw, bsb, bs_stage, nkc, c, 1, rs, bsi, rph, bph, acc1);
        acc[0] = acc1[0];
      } else {
        ok = dp4a_chunks<WQ4, MODE, TT, PK>(P, B, raw, bsb, bs_stage, nkc, c, nj, rs, bsi, rph, bph, acc);
      }
      if (!ok) break;
      if constexpr (MODE == kGateUp) {
        const int r = c & (RG - 1);
        if (up_row) {
          // Hand the up sums to the gate threads (bounded waits: a wait
          // that gives up raises the CTA's abort flag).
          if (!(ok = wait_bar(&B->xch_empty, xph ^ 1, B, P.err))) break;
#pragma unroll
          for (int t = 0; t < TT; ++t)
            if (t < nj) xch[t * RG + r] = acc[t];
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&B->xch_full);
          xph ^= 1;
          continue;
        }
        if (!(ok = wait_bar(&B->xch_full, xph, B, P.err))) break;
        float upv[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) upv[t] = t < nj ? xch[t * RG + r] : 0.f;
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&B->xch_empty);
        xph ^= 1;
        // act = gelu(gate) * up (ops.rs:99-114), then the down product's
        // Q8_0 re-quantisation (quant.rs:193-228): a warp's 32 lanes hold the
        // 32 elements of one act block.
        if (m0 + r - lane < P.rows) {
          const int blk = (m0 + r - lane) >> 5;
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            if (t < nj) {
              const float v = __fmul_rn(gelu_approx(acc[t]), upv[t]);
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
              const int pos = p0 + t;
              uint8_t* dst = reinterpret_cast<uint8_t*>(P.out_q) +
                             act_group_offset(true, blk, pos >> 3, P.out_nb, P.npad) + (lane >> 4) * 128 + (pos & 7) * 16 +
                             (lane & 15);
              *dst = (uint8_t)(int8_t)qv;
              if (lane == 0) {
                const int corr = P.down_q4 ? kMagicI - 8 * qsum : kMagicI;
                store_act_scale_gm(P.out_s, blk, pos, P.out_nb, f16_bits_to_f32(d16), corr);
              }
            }
          }
        }
      } else {
        const int ra = m0 + c;
        if (ra < P.rows) {
#pragma unroll
          for (int t = 0; t < TT; ++t)
            if (t < nj) P.y[(size_t)(p0 + t) * P.rows + ra] = acc[t];
        }
      }
    }
  }
}

}  // namespace gv

// ---------------------------------------------------------------- host side

namespace {

constexpr int kSmemLimit = 227 * 1024;

struct GvPlan {
  int rs, bs, raw_bytes, kcb, per_sm;
  size_t smem;
};

// Several CTAs per SM when there are more units than SMs, otherwise one CTA
// with as deep a weight ring as fits (few units: each SM must keep many bytes
// in flight on its own).
// Tuning overrides (mrml_moe_set_option): CTAs per SM and weight-ring depth
// of the decode kernel; 0 = automatic.
std::atomic<int> g_gv_per_sm{0}, g_gv_ring{0}, g_gv_per_sm_down{0};

GvPlan gv_plan(int mode, int wtype, int nb, int row_bytes, bool many_units, bool mma, int ng, bool packed = false,
               int per_sm_want = 0) {
  GvPlan p{};
  const int bb = block_bytes(wtype);
  // down on packed weights streams K chunks (down_chunk_blocks); on GGUF rows a whole K per unit
  p.kcb = mode == tc::kGateUp ? tc::kKC : (packed ? down_chunk_blocks(nb) : nb);
  const int raw1 = mode == tc::kGateUp ? 2 * kGvRowsGateUp * tc::kKC * bb
                                       : (packed ? 2 * kGvRowsGateUp * p.kcb * bb : 2 * kGvRowsGateUp * row_bytes);
  p.raw_bytes = (raw1 + 1023) & ~1023;
  const int bs_stage = p.kcb * ng * (256 + kActScaleBytes);
  const size_t xch_bytes = mode == tc::kGateUp ? (size_t)kGvTokens * ng * kGvRowsGateUp * 4 : 0;
  // With many units, as many CTAs per SM as fit with a double-buffered weight
  // ring (the kernel's launch bound, ctas_per_sm); with few units (at most
  // one per SM), the ring that fits a third of the SM's shared memory.
  // Measured on B200 at config 2, T = 1 (99 gate/up units): 42.4 us per layer
  // step against 45.2 us with one CTA's deepest ring (the whole SM).
  const int bound = gv::ctas_per_sm(mma, mode, ng, wtype == kQ4_0, packed);
  const int down_set = mode == tc::kGateUp ? 0 : g_gv_per_sm_down.load();
  const int per_sm_set = down_set > 0 ? down_set : g_gv_per_sm.load(), ring_set = g_gv_ring.load();
  const int per_sm_auto = per_sm_want > 0 ? std::min(per_sm_want, bound) : (many_units ? bound : std::min(bound, 3));
  const int per_sm_max = per_sm_set > 0 ? per_sm_set : per_sm_auto;
  for (int per_sm = per_sm_max; per_sm >= 1; --per_sm) {
    const size_t budget = kSmemLimit / per_sm - (per_sm > 1 ? 1024 : 0);
    // GGUF down tiles hold a whole K (one stage per unit); several CTAs per
    // SM overlap one another's loads, so a single stage each is allowed there.
    // K-chunked stages (gate/up, packed down) double-buffer within a CTA.
    const int rs_min = (per_sm > 1 && (mode == tc::kGateUp || packed)) ? 2 : 1;
    const int rs_max = ring_set > 0 ? ring_set : tc::kMaxRaw;
    for (int rs = rs_max; rs >= rs_min; --rs)
      for (int bs = 2; bs >= 1; --bs) {
        const size_t total = 128 + tc::kGvBarBytes + (size_t)rs * p.raw_bytes + (size_t)bs * bs_stage + xch_bytes;
        if (total <= budget) {
          p.rs = rs;
          p.bs = bs;
          p.smem = total;
          p.per_sm = per_sm;
          return p;
        }
      }
  }
  p.smem = 0;
  return p;
}

template <int WQ4, int MODE, int MMA, int NG, int PK>
cudaError_t gv_launch(const CUtensorMap& map, const tc::Params& P, size_t smem, int grid, cudaStream_t s) {
  auto kern = gv::moe_gemv_kernel<WQ4, MODE, MMA, NG, PK>;
  static SmemOptIn cache;
  const cudaError_t st = ensure_smem(kern, smem, cache);
  if (st != cudaSuccess) return st;
  return launch_pdl(kern, dim3(grid), dim3(32 * (gv::kComp0 + gv::kCompWarps)), smem, s, map, P);
}

}  // namespace

void gv_set_tuning(int per_sm, int ring, int per_sm_down) {
  g_gv_per_sm = per_sm;
  g_gv_ring = ring;
  g_gv_per_sm_down = per_sm_down;
}

bool gv_supported(int wtype, int H, int I) {
  if (H % 256 != 0 || I % 32 != 0) return false;
  const int down_row = (I / 32) * block_bytes(wtype);
  if (I % kGvRowsGateUp != 0) return false;
  if (gv_plan(tc::kGateUp, wtype, H / 32, 0, false, false, 1).smem == 0) return false;
  if (gv_plan(tc::kDown, wtype, I / 32, down_row, false, false, 1).smem == 0) return false;
  return tc_map_available();
}

bool gv_packed_supported(int wtype, int H, int I) {
  // gate/up groups of 64 rows and K chunks of kKC blocks; down groups of 128
  return gv_supported(wtype, H, I) && H % 128 == 0 && (H / 32) % tc::kKC == 0 && I % kGvRowsGateUp == 0;
}

bool gv_two_groups_supported(int wtype, int H, int I) {
  const int down_row = (I / 32) * block_bytes(wtype);
  return gv_plan(tc::kGateUp, wtype, H / 32, 0, true, true, 2).smem != 0 &&
         gv_plan(tc::kDown, wtype, I / 32, down_row, true, true, 2).smem != 0;
}

template <int PK>
cudaError_t gv_dispatch(int mode, bool q4, bool mma, int ng, const CUtensorMap& map, const tc::Params& P, size_t smem,
                        int grid, cudaStream_t s) {
  if (mma && ng == 2) {
    if (mode == tc::kGateUp)
      return q4 ? gv_launch<1, tc::kGateUp, 1, 2, PK>(map, P, smem, grid, s)
                : gv_launch<0, tc::kGateUp, 1, 2, PK>(map, P, smem, grid, s);
    return q4 ? gv_launch<1, tc::kDown, 1, 2, PK>(map, P, smem, grid, s)
              : gv_launch<0, tc::kDown, 1, 2, PK>(map, P, smem, grid, s);
  }
  if (mma) {
    if (mode == tc::kGateUp)
      return q4 ? gv_launch<1, tc::kGateUp, 1, 1, PK>(map, P, smem, grid, s)
                : gv_launch<0, tc::kGateUp, 1, 1, PK>(map, P, smem, grid, s);
    return q4 ? gv_launch<1, tc::kDown, 1, 1, PK>(map, P, smem, grid, s)
              : gv_launch<0, tc::kDown, 1, 1, PK>(map, P, smem, grid, s);
  }
  if (mode == tc::kGateUp)
    return q4 ? gv_launch<1, tc::kGateUp, 0, 1, PK>(map, P, smem, grid, s)
              : gv_launch<0, tc::kGateUp, 0, 1, PK>(map, P, smem, grid, s);
  return q4 ? gv_launch<1, tc::kDown, 0, 1, PK>(map, P, smem, grid, s)
            : gv_launch<0, tc::kDown, 0, 1, PK>(map, P, smem, grid, s);
}

cudaError_t launch_gemv(int mode, int wtype, bool packed, bool mma, int ng, const uint8_t* weights, int H, int I,
                        int E, const int8_t* bq, const int2* bsc, const int4* units, const int* n_units, int max_units,
                        int npad, int8_t* out_q, int2* out_s, float* y, int* err, cudaStream_t s, int per_sm) {
  if (ng != 1 && !(ng == 2 && mma)) return cudaErrorInvalidValue;
  if (packed && !gv_packed_supported(wtype, H, I)) return cudaErrorInvalidValue;
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
  const int sms = tc_num_sms();
  const bool many = max_units > sms;
  GvPlan pl;
  if (mode == tc::kGateUp) {
    P.nb = H / 32;
    P.rows = I;
    P.row_bytes = (H / 32) * bb;
    P.out_q = out_q;
    P.out_s = out_s;
    P.out_nb = I / 32;
    P.down_q4 = wtype == kQ4_0;
    if (packed)
      P.w_raw = weights;
    else if (!tc_make_gate_up_map(&map, weights, wtype, H, I, E, kGvRowsGateUp))
      return cudaErrorInvalidValue;
    pl = gv_plan(mode, wtype, P.nb, P.row_bytes, many, mma, ng, packed, per_sm);
  } else {
    P.nb = I / 32;
    P.rows = H;
    P.row_bytes = (I / 32) * bb;
    P.w_raw = weights;
    P.y = y;
    pl = gv_plan(mode, wtype, P.nb, P.row_bytes, many, mma, ng, packed, per_sm);
  }
  if (pl.smem == 0) return cudaErrorInvalidValue;
  P.rs = pl.rs;
  P.bs = pl.bs;
  P.raw_bytes = pl.raw_bytes;
  P.kcb = pl.kcb;
  P.one = 1.0f;
  const int grid = std::max(1, std::min(pl.per_sm * sms, max_units));
  const bool q4 = wtype == kQ4_0;
  return packed ? gv_dispatch<1>(mode, q4, mma, ng, map, P, pl.smem, grid, s)
                : gv_dispatch<0>(mode, q4, mma, ng, map, P, pl.smem, grid, s);
}

}  // namespace mrml
