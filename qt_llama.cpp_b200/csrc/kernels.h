// kernels.h — host launchers of the MRML MoE kernels (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrml {

cudaError_t launch_router_logits(const float* W, const float* x, float* logits, float* bounds, int H, int E, int T,
                                 cudaStream_t s);
cudaError_t launch_router_topk(const float* W, const float* x, float* logits, const float* bounds, int32_t* ids,
                               float* probs, int H, int E, int K, int T, int* stats, cudaStream_t s);
cudaError_t launch_quantize_rows(const float* x, int8_t* xq, float* xd, int32_t* xsum, long long n_blocks,
                                 cudaStream_t s);
cudaError_t launch_quantize_gguf(int wtype, const float* x, uint8_t* dst, long long n_blocks, cudaStream_t s);
cudaError_t launch_dispatch(const int32_t* ids, const float* probs, int n_pairs, int E, int32_t* offsets,
                            int32_t* sorted, int32_t* pos, int* err, cudaStream_t s);
cudaError_t launch_gate_up(int wtype, const uint8_t* gate_up, const int32_t* offsets, const int32_t* sorted,
                           const int8_t* xq, const float* xd, const int32_t* xsum, float* act, int H, int I, int E,
                           int K, int* err, cudaStream_t s);
cudaError_t launch_down(int wtype, const uint8_t* down, const int32_t* offsets, const float* act, float* ydown, int H,
                        int I, int E, int* err, cudaStream_t s);
cudaError_t launch_combine(const float* ydown, const int32_t* pos, const int32_t* ids, const float* probs,
                           const float* down_scale, float* out, int H, int K, int T, cudaStream_t s);
int gate_up_tok_chunk(int wtype, int H);
int down_tok_chunk(int wtype, int I);

}  // namespace mrml
