// pipe.cuh — building blocks of the warp-specialised expert kernels
// (gemm_tc.cu on the tensor cores, gemv.cu on the CUDA cores): the work-unit
// parameters, the mbarrier set, bounded waits, TMA copies, the tcgen05
// descriptors and the raw GGUF block readers.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mrml {
namespace tc {

constexpr int kM = 128;        // weight rows per tile (MMA M)
constexpr int kKC = 8;         // quant blocks per gate/up K chunk (8*18 and 8*34 bytes are 16-byte multiples)
constexpr int kConvWarps = 4;
constexpr int kConvWarp0 = 3;
constexpr int kEpiWarp0 = 7;
constexpr int kMaxRing = 16;

enum Mode : int { kGateUp = 0, kDown = 1 };

struct Params {
  const uint8_t* w_raw;  // down: raw weights [E][rows][row_bytes]
  const int8_t* bq;      // B operand [nb][npad_alloc/8][2][8][16]
  const int2* bsc;       // B scales: [nb][npad_alloc] {f32 bits of d_a, int32 correction}
                         // (tensor cores), group-major records (decode kernel)
  const int4* units;     // {e, p0, nvalid, m0}
  const int* n_units;
  int nb;                // quant blocks along K
  int rows;              // weight rows per expert part (I for gate/up, H for down)
  int row_bytes;         // raw bytes per weight row
  int npad;              // position stride of bq/bsc/out (npad_alloc)
  int w_q4;              // 1: weights Q4_0 (unsigned nibbles), 0: Q8_0
  // gate/up outputs: act as the down product's B operand and its scales
  int8_t* out_q;
  int2* out_s;
  int down_q4;           // the down weights' type (selects the act correction)
  int out_nb;            // quant blocks per act row (I / 32), group-major act layout
  // down output
  float* y;              // [npad_alloc][H]
  int* err;
  // ring sizes
  int rs, as, bs, tb;
  int raw_bytes;         // bytes per raw stage
  int kcb;               // blocks per B stage (kKC for gate/up, nb for down)
  float one;             // 1.0f, opaque to the compiler (decode kernel's chain adds)
};

constexpr int kMaxRaw = 8;

struct __align__(8) Bars {
  uint64_t raw_full[kMaxRaw], raw_empty[kMaxRaw];
  uint64_t conv_full[kMaxRing], conv_empty[kMaxRing];   // A-tile ring (freed by the MMA's commit)
  uint64_t dw_full[kMaxRing], dw_empty[kMaxRing];       // weight-scale ring, one slot per TMEM slot
  uint64_t bs_full[4], bs_empty[4];
  uint64_t tmem_full[kMaxRing], tmem_empty[kMaxRing];
  uint64_t xch_full, xch_empty;  // gate/up row exchange of the CUDA-core kernel
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(Bars) <= 1024, "the barrier block must fit the first KiB of shared memory");

// The decode kernel's barrier block: only the rings it uses, so that five
// of its CTAs fit an SM's shared memory with both activation stages.
struct __align__(8) GvBars {
  uint64_t raw_full[kMaxRaw], raw_empty[kMaxRaw];
  uint64_t bs_full[4], bs_empty[4];
  uint64_t xch_full, xch_empty;
  int abort;
};
constexpr int kGvBarBytes = 256;
static_assert(sizeof(GvBars) <= kGvBarBytes, "the decode barrier block must fit its 256 bytes");

template <class BarsT>
__device__ __forceinline__ bool aborted(const BarsT* B) { return *(const volatile int*)&B->abort != 0; }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also watches the CTA's abort flag.
template <class BarsT>
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, BarsT* B, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && aborted(B)) return false;
    if (i > 128) __nanosleep(64);
  }
  set_error(err, kDevTimeout);
  *(volatile int*)&B->abort = 1;
  return false;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, canonical K-major layout without swizzle:
// 8-row x 16-byte core matrices stored contiguously; LBO = distance between
// the two core matrices along K (128 B), SBO = distance between 8-row groups
// (256 B).  Bits 46-47 hold the descriptor version (1) for sm_100.
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint32_t a = smem_u32(p);
  uint64_t d = (uint64_t)((a >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 16;
  d |= (uint64_t)(256 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8: D s32, A u8 or s8,
// B s8, both K-major, N and M encoded as N>>3 and M>>4.
__host__ __device__ constexpr uint32_t idesc_i8(bool a_unsigned, int N, int M) {
  return (2u << 4) | ((a_unsigned ? 0u : 1u) << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- convert
// Writes one row's 32 int8 values (two 16-byte halves) into an A tile in the
// canonical layout: core (g, c) at (2g + c)*128, row rr at +16*rr.
__device__ __forceinline__ void store_a_row(int8_t* tile, int r, uint4 lo, uint4 hi) {
  uint8_t* base = reinterpret_cast<uint8_t*>(tile) + (r >> 3) * 256 + (r & 7) * 16;
  *reinterpret_cast<uint4*>(base) = lo;
  *reinterpret_cast<uint4*>(base + 128) = hi;
}

// Q4_0 block -> unsigned nibble bytes: low nibbles are elements 0..15,
// high nibbles elements 16..31 (quant.rs:119-163).
__device__ __forceinline__ void q4_to_a(const uint32_t (&qs)[4], uint4& lo, uint4& hi) {
  lo = make_uint4(qs[0] & 0x0f0f0f0fu, qs[1] & 0x0f0f0f0fu, qs[2] & 0x0f0f0f0fu, qs[3] & 0x0f0f0f0fu);
  hi = make_uint4((qs[0] >> 4) & 0x0f0f0f0fu, (qs[1] >> 4) & 0x0f0f0f0fu, (qs[2] >> 4) & 0x0f0f0f0fu,
                  (qs[3] >> 4) & 0x0f0f0f0fu);
}

// Reads the 16-byte-aligned window around block `bl` of a gate/up chunk row
// (row pitch 8*BB bytes, a 16-byte multiple) and extracts the block.
template <int BB, int BL>
__device__ __forceinline__ void chunk_block(const uint8_t* row, uint32_t& d16, uint32_t (&qs)[BB == 18 ? 4 : 8]) {
  constexpr int start = BB * BL;
  constexpr int w0 = (start & ~15);
  constexpr int nvec = ((start + BB - w0) + 15) / 16;
  uint32_t w[4 * nvec];
#pragma unroll
  for (int v = 0; v < nvec; ++v) {
    const uint4 t = *reinterpret_cast<const uint4*>(row + w0 + 16 * v);
    w[4 * v] = t.x;
    w[4 * v + 1] = t.y;
    w[4 * v + 2] = t.z;
    w[4 * v + 3] = t.w;
  }
  constexpr int off = start - w0;  // even, 0..14
  constexpr int wi = off / 4;
  if constexpr ((off & 3) == 0) {  // scale in the low half of w[wi]
    d16 = w[wi] & 0xffffu;
#pragma unroll
    for (int i = 0; i < (BB == 18 ? 4 : 8); ++i) qs[i] = __funnelshift_r(w[wi + i], w[wi + i + 1], 16);
  } else {  // scale in the high half, values word-aligned
    d16 = w[wi] >> 16;
#pragma unroll
    for (int i = 0; i < (BB == 18 ? 4 : 8); ++i) qs[i] = w[wi + 1 + i];
  }
}


}  // namespace tc
}  // namespace mrml
