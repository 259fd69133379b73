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

// tanh for the GeGLU epilogue: the double-precision libdevice tanh rounded
// once to f32.  It equals the correctly rounded f32 tanh except in rare
// double-rounding cases; glibc's tanhf (the reference) is within about one
// ulp of that.
__device__ __forceinline__ float tanh_f32(float x) { return (float)tanh((double)x); }

// ops.rs:101-104, evaluated left to right without contraction:
// 0.5*x*(1 + tanh(0.7978845608*(x + 0.044715*x*x*x))).
__device__ __forceinline__ float gelu_approx(float x) {
  float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, cube));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanh_f32(inner)));
}

// expf for the router softmax: double exp rounded once to f32 (equal to the
// correctly rounded expf except in rare double-rounding cases).
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }

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

// Activation operand layouts (quantised Q8_0 rows by position).  Positions
// come in groups of 8; a group's block b is 256 bytes: two 16-byte halves
// (elements 0..15 at +0, 16..31 at +128) of 8 positions (16 bytes apart),
// the canonical no-swizzle K-major core matrices of a tcgen05 B operand.
//  - block-major (tensor cores): group g of block b at (b * npad/8 + g) * 256,
//    so a block's token tile is contiguous; scales at [b * npad + pos].
//  - group-major (decode kernel): at (g * nb + b) * 256, so a group's
//    consecutive blocks are contiguous; scales at [(g * nb + b) * 8 + pos % 8].
__host__ __device__ inline size_t act_group_offset(bool group_major, int b, int g, int nb, int npad) {
  return group_major ? ((size_t)g * nb + b) * 256 : ((size_t)b * (npad / 8) + g) * 256;
}
__host__ __device__ inline size_t act_scale_index(bool group_major, int b, int pos, int nb, int npad) {
  return group_major ? ((size_t)(pos >> 3) * nb + b) * 8 + (pos & 7) : (size_t)b * npad + pos;
}

}  // namespace mrml
