// prepare.cu — load-time repack of GGUF expert weights into the decode
// kernel's packed layout (mrml_moe_prepare_weights).
//
// The reference uploads the GGUF expert slabs unchanged (model.rs:726-741):
// gate_up [E][2I][H/32] blocks, down [E][H][I/32] blocks of 18 bytes (Q4_0:
// f16 scale, 16 nibble bytes) or 34 bytes (Q8_0: f16 scale, 32 int8).  A
// block's values start 2 bytes past its start, so in shared memory half of
// them sit 2 bytes off a word boundary, and the decode kernel's warp-level
// MMA needs one row's 4-byte piece per lane from two rows at once.  The
// packed layout keeps every byte (same size) but orders them by MMA fragment:
//
//   record (16-row tile, block), 16 * block_bytes long:
//     Q4_0: lane l = 4g + t owns bytes [8l, 8l+8): the raw nibble bytes
//           [4t, 4t+4) of tile rows g and g+8; then 16 f16 scales as pairs
//           {d(g), d(g+8)} at 256 + 4g;
//     Q8_0: lane l owns bytes [16l, 16l+16): rows g, g+8 values [4t, 4t+4),
//           then rows g, g+8 values [16+4t, 16+4t+4); scales at 512 + 4g.
//   gate_up: [E][part: gate rows, up rows][64-row group][K chunk of 8
//            blocks][tile 4][block 8][record]  (a unit's K chunk is one
//            contiguous run per part);
//   down:    [E][128-row group][K chunk of down_chunk_blocks(I/32) blocks]
//            [tile 8][block][record]  (a unit's K chunk is one contiguous
//            run).
//
// The values are the reference's bytes; only their order changes, so the
// products are bit-identical to the raw layout's.
#include "../../include/mrml_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace mrml {

// One thread per (expert, row, block).
template <int WQ4>
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int which, int rows_part,
                              int parts, int nb, long long n) {
  constexpr int BB = WQ4 ? 18 : 34, RB = 16 * BB, NW = WQ4 ? 4 : 8;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int b = (int)(i % nb);
  const long long er = i / nb;                  // expert * (parts * rows_part) + row
  const int rows = parts * rows_part;
  const int e = (int)(er / rows), rall = (int)(er % rows);
  const int p = rall / rows_part, r = rall % rows_part;
  const uint16_t* blk = reinterpret_cast<const uint16_t*>(src + (size_t)i * BB);  // 2-byte aligned
  uint32_t w[NW];
#pragma unroll
  for (int k = 0; k < NW; ++k) w[k] = (uint32_t)blk[1 + 2 * k] | ((uint32_t)blk[2 + 2 * k] << 16);
  const uint16_t d16 = blk[0];
  size_t rec;
  if (which == 0) {  // gate_up: 64-row groups, K chunks of 8 blocks, 4 tiles
    const int nG = rows_part / 64, nC = nb / 8;
    const int G = r / 64, j = (r % 64) / 16, c = b / 8, bl = b % 8;
    rec = (((((size_t)e * parts + p) * nG + G) * nC + c) * 4 + j) * 8 + bl;
  } else {  // down: 128-row groups, K chunks of down_chunk_blocks(nb) blocks, 8 tiles
    const int nG = rows_part / 128, kc = down_chunk_blocks(nb), nC = nb / kc;
    const int G = r / 128, j = (r % 128) / 16, c = b / kc, bl = b % kc;
    rec = ((((size_t)e * nG + G) * nC + c) * 8 + j) * kc + bl;
  }
  uint8_t* out = dst + rec * RB;
  const int rr = r % 16, g = rr & 7, h = rr >> 3;
  if constexpr (WQ4) {
#pragma unroll
    for (int t = 0; t < 4; ++t) *reinterpret_cast<uint32_t*>(out + 8 * (4 * g + t) + 4 * h) = w[t];
    *reinterpret_cast<uint16_t*>(out + 256 + 4 * g + 2 * h) = d16;
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      *reinterpret_cast<uint32_t*>(out + 16 * (4 * g + t) + 4 * h) = w[t];
      *reinterpret_cast<uint32_t*>(out + 16 * (4 * g + t) + 8 + 4 * h) = w[4 + t];
    }
    *reinterpret_cast<uint16_t*>(out + 512 + 4 * g + 2 * h) = d16;
  }
}

cudaError_t launch_repack(int which, int wtype, const uint8_t* src, uint8_t* dst, int H, int I, int E,
                          cudaStream_t s) {
  const int rows_part = which == 0 ? I : H, parts = which == 0 ? 2 : 1, nb = (which == 0 ? H : I) / 32;
  const long long n = (long long)E * parts * rows_part * nb;
  const int blocks = (int)((n + 255) / 256);
  if (wtype == kQ4_0)
    repack_kernel<1><<<blocks, 256, 0, s>>>(src, dst, which, rows_part, parts, nb, n);
  else
    repack_kernel<0><<<blocks, 256, 0, s>>>(src, dst, which, rows_part, parts, nb, n);
  return cudaPeekAtLastError();
}

}  // namespace mrml
