// common.cuh — shared device helpers for the MRML MoE kernels (sm_100a).
//
// Floating-point rule for this library: every operation that must agree bit
// for bit with the reference CPU path is written with an explicit
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn) so that nvcc
// cannot contract it into an FMA.  The reference Rust code never fuses.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrml {

constexpr int kQ4_0 = 2;  // GGML type ids, crates/mrml-tensor/src/types.rs:7-27
constexpr int kQ8_0 = 8;

// Device-side status codes written to the error word.
constexpr int kDevOk = 0;
constexpr int kDevTimeout = 1;      // a bounded wait gave up
constexpr int kDevBadExpert = 2;    // an expert id outside [0, E)
constexpr int kDevOverflow = 3;     // a size that exceeds a compiled limit

// Iteration limit for every spin wait in this library (~1 s at 2 GHz with
// the nanosleep back-off below).
constexpr uint32_t kSpinLimit = 1u << 24;

// 1.5 * 2^23: adding an integer n with |n| < 2^22 to these bits gives the
// float 1.5*2^23 + n exactly, so (bits + n) - kMagicF == (float)n.
constexpr int32_t kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

// Programmatic dependent launch (launch_pdl): wait for the previous grid on
// the stream (a no-op when launched without the attribute), and let the
// next grid start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// quant.rs:47-77: f16 bits -> f32, subnormals expanded.  The hardware
// conversion is exact for every f16 value, including subnormals.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// quant.rs:81-104: truncating f32 -> f16 bits, exponent underflow -> +0.
__device__ __forceinline__ uint32_t f32_to_f16_trunc(float f) {
  uint32_t bits = __float_as_uint(f);
  uint32_t sign = (bits >> 31) & 1u;
  int32_t exp = (int32_t)((bits >> 23) & 0xffu);
  uint32_t mant = bits & 0x7fffffu;
  if (exp == 255) return (sign << 15) | (mant == 0 ? 0x7c00u : 0x7e00u);
  int32_t exp16 = exp - 127 + 15;
  if (exp16 >= 31) return (sign << 15) | 0x7c00u;
  if (exp16 <= 0) return 0u;
  return (sign << 15) | ((uint32_t)exp16 << 10) | (mant >> 13);
}

// dp4a with unsigned bytes in `a` (Q4_0 nibbles 0..15) and signed bytes in
// `b` (Q8_0 activations).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// tanh for the GeGLU epilogue, bit-identical to the reference's: the Rust
// reference's f32::tanh is the C library's tanhf, which in glibc 2.39 is the
// fdlibm single-precision algorithm (sysdeps/ieee754/flt-32/s_tanhf.c and
// s_expm1f.c).  That algorithm is restated here step for step in f32 with
// round-to-nearest operations and no contraction:
//   tanh(x) = sign(x) * (|x| >= 1 ? 1 - 2 / (expm1(2|x|) + 2)
//                                 : -m / (m + 2), m = expm1(-2|x|)),
//   x for |x| < 2^-55 (as x * (1 + x)), 1 for |x| >= 22;
//   expm1(x): x = k ln2 + r (ln2 split hi/lo, compensation c), then
//   r - (r*e - r^2/2) with e from the Remez rational approximation
//   R1 = 1 + hxs*(Q1 + hxs*(Q2 + ... Q5)), hxs = r^2/2, and reconstruction
//   by the exponent k.
// The steps are evaluated for every input and the case is chosen by
// selects (the case split depends on the data, and branches would diverge
// inside a warp); every case computes exactly glibc's operations.  This
// form was checked equal to glibc's tanhf on all 2^32 - 2^24 + 2 non-NaN
// f32 inputs.
namespace tanh_glibc {
constexpr float kLn2Hi = 6.9313812256e-01f, kLn2Lo = 9.0580006145e-06f, kInvLn2 = 1.4426950216e+00f;
constexpr float kQ1 = -3.3333335072e-02f, kQ2 = 1.5873016091e-03f, kQ3 = -7.9365076090e-05f,
                kQ4 = 4.0082177293e-06f, kQ5 = -2.0109921195e-07f;

// expm1 for finite |x| < 44 (other inputs give unused garbage).
__device__ __forceinline__ float expm1(float x) {
  const uint32_t ax = __float_as_uint(x) & 0x7fffffffu;
  const bool neg = (__float_as_uint(x) >> 31) != 0;
  // Reduction x = k ln2 + (hi - lo); k = 0 (no reduction) for |x| <= ln2/2,
  // +-1 up to 1.5 ln2, else round(x / ln2).  k = 0 and k = +-1 give the
  // same values as glibc's special-cased forms.
  int k = 0;
  if (ax > 0x3eb17218u) {
    const int kg = __float2int_rz(__fadd_rn(__fmul_rn(kInvLn2, x), neg ? -0.5f : 0.5f));
    k = ax < 0x3f851592u ? (neg ? -1 : 1) : kg;
  }
  const float tk = (float)k;
  const float hi = __fsub_rn(x, __fmul_rn(tk, kLn2Hi));
  const float lo = __fmul_rn(tk, kLn2Lo);
  const float xr = __fsub_rn(hi, lo);
  const float c = __fsub_rn(__fsub_rn(hi, xr), lo);
  const float hfx = __fmul_rn(0.5f, xr);
  const float hxs = __fmul_rn(xr, hfx);
  float r1 = __fadd_rn(kQ4, __fmul_rn(hxs, kQ5));
  r1 = __fadd_rn(kQ3, __fmul_rn(hxs, r1));
  r1 = __fadd_rn(kQ2, __fmul_rn(hxs, r1));
  r1 = __fadd_rn(kQ1, __fmul_rn(hxs, r1));
  r1 = __fadd_rn(1.0f, __fmul_rn(hxs, r1));
  const float t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
  float e = __fmul_rn(hxs, __fdiv_rn(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(xr, t))));
  const float res0 = __fsub_rn(xr, __fsub_rn(__fmul_rn(xr, e), hxs));  // k == 0
  e = __fsub_rn(__fsub_rn(__fmul_rn(xr, __fsub_rn(e, c)), c), hxs);
  const float resm1 = __fsub_rn(__fmul_rn(0.5f, __fsub_rn(xr, e)), 0.5f);  // k == -1
  const float res1 = xr < -0.25f ? __fmul_rn(-2.0f, __fsub_rn(e, __fadd_rn(xr, 0.5f)))
                                 : __fadd_rn(1.0f, __fmul_rn(2.0f, __fsub_rn(xr, e)));  // k == 1
  const uint32_t kb = (uint32_t)k << 23;
  // k <= -2 or k > 56: 2^k * (1 - (e - x)) - 1
  const float resA = __fsub_rn(__uint_as_float(__float_as_uint(__fsub_rn(1.0f, __fsub_rn(e, xr))) + kb), 1.0f);
  // 2 <= k < 23: 2^k * ((1 - 2^-k) - (e - x))
  const int ks = min(max(k, 2), 22);
  const float resB = __uint_as_float(
      __float_as_uint(__fsub_rn(__uint_as_float(0x3f800000u - (0x1000000u >> ks)), __fsub_rn(e, xr))) + kb);
  // 23 <= k <= 56: 2^k * ((x - (e + 2^-k)) + 1)
  const int kc = min(max(k, 23), 56);
  const float resC = __uint_as_float(
      __float_as_uint(__fadd_rn(__fsub_rn(xr, __fadd_rn(e, __uint_as_float((uint32_t)(0x7f - kc) << 23))), 1.0f)) +
      kb);
  float r = k == 0    ? res0
            : k == -1 ? resm1
            : k == 1  ? res1
            : (k <= -2 || k > 56) ? resA
            : k < 23  ? resB
                      : resC;
  if (ax < 0x33000000u) r = x;                                        // |x| < 2^-25
  if (ax >= 0x4195b844u && neg) r = __fsub_rn(1.0e-30f, 1.0f);        // x < -27 ln2
  return r;
}
}  // namespace tanh_glibc

__device__ __forceinline__ float tanh_f32(float x) {
  const uint32_t ax = __float_as_uint(x) & 0x7fffffffu;
  const bool big = ax >= 0x3f800000u;  // |x| >= 1
  const float a = fabsf(x);
  const float m = tanh_glibc::expm1(big ? __fmul_rn(2.0f, a) : __fmul_rn(-2.0f, a));
  // |x| >= 1: 1 - 2 / (m + 2);  |x| < 1: -m / (m + 2)
  const float q = __fdiv_rn(big ? 2.0f : -m, __fadd_rn(m, 2.0f));
  float z = big ? __fsub_rn(1.0f, q) : q;
  if (ax >= 0x41b00000u) z = 1.0f;  // |x| >= 22: 1 - 1e-30 rounded
  z = (__float_as_uint(x) >> 31) ? -z : z;
  if (ax < 0x24000000u) z = __fmul_rn(x, __fadd_rn(1.0f, x));  // |x| < 2^-55 (and +-0)
  if (ax > 0x7f800000u) z = x;                                 // NaN
  return z;
}

// ops.rs:101-104, evaluated left to right without contraction:
// 0.5*x*(1 + tanh(0.7978845608*(x + 0.044715*x*x*x))).
__device__ __forceinline__ float gelu_approx(float x) {
  float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, cube));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanh_f32(inner)));
}

// expf for the router softmax, bit-identical to the reference's f32::exp,
// i.e. glibc 2.39's expf (sysdeps/ieee754/flt-32/e_expf.c, the table-driven
// algorithm published in ARM's optimized-routines): in double precision,
//   z = x * 32/ln2 = k + r  (k by the 1.5*2^52 shift trick, r in [-1/2, 1/2]),
//   2^(k/32) = s from a 32-entry table of 2^(i/32) (bits minus i*2^52/32)
//   with the exponent k>>5 added to the bits,
//   exp(x) ~= s * (C0 r^3 + C1 r^2 + C2 r + 1), rounded once to f32.
// glibc's x86-64 build contracts the multiply-adds into FMAs (the variant
// picked on FMA hardware, as on the B200 hosts); the steps below use the same
// fused operations.  Checked equal to glibc's expf on every f32 input in
// (-103.97, 88.72); outside it the result is 0 or +inf as in glibc.
namespace exp_glibc {
__device__ __constant__ const uint64_t kTab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};
constexpr double kInvLn2N = 0x1.71547652b82fep+0 * 32, kShift = 0x1.8p+52;
constexpr double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 kC2 = 0x1.62e42ff0c52d6p-1 / 32;
}  // namespace exp_glibc

__device__ __forceinline__ float exp_f32(float x) {
  using namespace exp_glibc;
  const uint32_t ux = __float_as_uint(x);
  if (((ux >> 20) & 0x7ffu) >= 0x42bu) {  // |x| >= 88 or not finite
    if (ux == 0xff800000u) return 0.0f;
    if (((ux >> 20) & 0x7ffu) >= 0x7f8u) return x + x;
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p6f) return 0.0f;
  }
  const double xd = (double)x;
  double kd = __fma_rn(kInvLn2N, xd, kShift);
  const uint64_t ki = (uint64_t)__double_as_longlong(kd);
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const double s = __longlong_as_double((long long)(kTab[ki % 32] + (ki << 47)));
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, r2, y);
  return __double2float_rn(__dmul_rn(y, s));
}

// C roundf: nearest integer, halfway cases away from zero (CUDA's roundf has
// these semantics).
__device__ __forceinline__ float round_half_away(float x) { return roundf(x); }

// ------------------------------------------------------------ mbarrier ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records a timeout
// in *err) if the phase does not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
  }
  set_error(err, kDevTimeout);
  return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted in bytes on
// `bar`.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Prefetch a global range into L2 (no completion tracking).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ------------------------------------------------------- block loaders ---
// Read one quant block of a row staged in shared memory.  Blocks are 18 B
// (Q4_0) or 34 B (Q8_0) and start at 2-byte alignment, so the loader reads
// the aligned words that cover the block and funnel-shifts when needed.
// `p` points at the block's first byte (the f16 scale).  The staging buffer
// must extend at least 4 bytes past the last block.
struct Q4Block {
  uint32_t d16;
  uint32_t qs[4];
};
struct Q8Block {
  uint32_t d16;
  uint32_t qs[8];
};

__device__ __forceinline__ Q4Block load_q4_block(const uint8_t* p) {
  const uintptr_t addr = (uintptr_t)p;
  const uint32_t* w = (const uint32_t*)(addr & ~(uintptr_t)3);
  Q4Block b;
  if (addr & 2) {  // scale in the high half of w[0], qs word-aligned
    b.d16 = w[0] >> 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) b.qs[i] = w[i + 1];
  } else {
    uint32_t W[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) W[i] = w[i];
    b.d16 = W[0] & 0xffffu;
#pragma unroll
    for (int i = 0; i < 4; ++i) b.qs[i] = __funnelshift_r(W[i], W[i + 1], 16);
  }
  return b;
}

__device__ __forceinline__ Q8Block load_q8_block(const uint8_t* p) {
  const uintptr_t addr = (uintptr_t)p;
  const uint32_t* w = (const uint32_t*)(addr & ~(uintptr_t)3);
  Q8Block b;
  if (addr & 2) {
    b.d16 = w[0] >> 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) b.qs[i] = w[i + 1];
  } else {
    uint32_t W[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) W[i] = w[i];
    b.d16 = W[0] & 0xffffu;
#pragma unroll
    for (int i = 0; i < 8; ++i) b.qs[i] = __funnelshift_r(W[i], W[i + 1], 16);
  }
  return b;
}

__host__ __device__ constexpr int block_bytes(int wtype) { return wtype == kQ4_0 ? 18 : 34; }

// Blocks per K chunk of the packed down weights (the decode kernel's down
// stages; nb = I / 32): the largest divisor of nb up to 12, so that a unit's
// rows stream in a few equal chunks (config 2: 22 = 2 x 11).
__host__ __device__ constexpr int down_chunk_blocks(int nb) {
  int c = nb < 12 ? nb : 12;
  while (c > 1 && nb % c != 0) --c;
  return c < 1 ? 1 : c;
}

// Activation operand layouts (quantised Q8_0 rows by position).  Positions
// come in groups of 8; a group's block b is 256 bytes: two 16-byte halves
// (elements 0..15 at +0, 16..31 at +128) of 8 positions (16 bytes apart),
// the canonical no-swizzle K-major core matrices of a tcgen05 B operand.
//  - block-major (tensor cores): group g of block b at (b * npad/8 + g) * 256,
//    so a block's token tile is contiguous; scales at [b * npad + pos].
//  - group-major (decode kernel): at (g * nb + b) * 256, so a group's
//    consecutive blocks are contiguous; scales in kActScaleBytes records at
//    (g * nb + b) * kActScaleBytes (act_scale_offset_gm).
// Block-major scales are int2 {d, correction} per position.
__host__ __device__ inline size_t act_group_offset(bool group_major, int b, int g, int nb, int npad) {
  return group_major ? ((size_t)g * nb + b) * 256 : ((size_t)b * (npad / 8) + g) * 256;
}
__host__ __device__ inline size_t act_scale_index(int b, int pos, int npad) { return (size_t)b * npad + pos; }

// Group-major scale record of (position group, block), 128 bytes: for each
// position pair (2t, 2t+1), t = 0..3,
//   at 16t:      float {d(2t), d(2t+1), d(2t), d(2t+1)}
//   at 64 + 16t: int   {c(2t), c(2t+1), c(2t), c(2t+1)}
// The decode kernel's m16n8k32 MMA gives lane t the block sums of rows g and
// g+8 at columns 2t and 2t+1 in accumulator registers (row g: 2t, 2t+1; row
// g+8: 2t, 2t+1); its f32 chain runs on those column pairs with packed f32x2
// operations, so it reads the pair's d values with one 8-byte load, and the
// MMA's accumulator seeds (rows g and g+8 x columns 2t, 2t+1) as one 16-byte
// load.  16 bytes per position.
constexpr int kActScaleBytes = 128;
__host__ __device__ inline size_t act_scale_offset_gm(int b, int pos, int nb) {
  return ((size_t)(pos >> 3) * nb + b) * kActScaleBytes;
}
__device__ __forceinline__ void store_act_scale_gm(void* base, int b, int pos, int nb, float d, int corr) {
  uint8_t* rec = static_cast<uint8_t*>(base) + act_scale_offset_gm(b, pos, nb);
  const int j = pos & 7, t = j >> 1, k = j & 1;
  float* dd = reinterpret_cast<float*>(rec) + 4 * t + k;
  dd[0] = d;
  dd[2] = d;
  int* c = reinterpret_cast<int*>(rec + 64) + 4 * t + k;
  c[0] = corr;
  c[2] = corr;
}
// d and correction of position j (0..7) of a record.
__device__ __forceinline__ float act_rec_d(const uint8_t* rec, int j) {
  return reinterpret_cast<const float*>(rec)[4 * (j >> 1) + (j & 1)];
}
__device__ __forceinline__ int act_rec_corr(const uint8_t* rec, int j) {
  return reinterpret_cast<const int*>(rec + 64)[4 * (j >> 1) + (j & 1)];
}

}  // namespace mrml
