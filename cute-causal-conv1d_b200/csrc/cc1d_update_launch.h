// Argument blocks and host entry points of the update and varlen-state kernels.
#pragma once

#include <cuda_runtime.h>

#include "cc1d_common.cuh"

namespace cc1d {

constexpr int kUpdateRows = 4;  // batch rows per thread in the update kernel

struct UpdateArgs {
  int64_t batch, dim, seqlen, state_len;
  int64_t state_batch;  // rows of conv_state: a gather index outside [0, state_batch) is a padding row
  TensorArg x, state, weight, bias, out;
  const int32_t* cache_seqlens;  // nullable
  int64_t cache_stride;
  const int32_t* indices;        // nullable
  int64_t indices_stride;
  int32_t silu;
  int32_t weight_vec;  // weight is contiguous fp32 (dim, W), 16-byte aligned, and packets are used
                      // (update_shift_kernel: contiguous fp32 (dim, W), 16-byte aligned)
  int32_t bias_vec;    // decode kernels: bias is contiguous fp32, 16-byte aligned
};

// Single-token decode kernels (cc1d_decode.cu), by conv_state layout.
constexpr int kDecodeClShift = 0;  // channels contiguous, shift update (state_len == W-1)
constexpr int kDecodeClCirc = 1;   // channels contiguous, circular buffer
constexpr int kDecodeBlock = 2;    // (B, D, W-1) with entries contiguous, shift update
constexpr int kDecodeRing = 3;     // (B, D, S) with entries contiguous, circular, 16-bit, S % 4 == 0

struct VarlenArgs {
  int64_t batch, dim, state_len;
  int64_t total_tokens;  // rows of x: a gathered row at or past the end gives zeros
  TensorArg x, states;  // x: (tokens, dim) strides s0, s1 ; states: (batch, dim, state_len)
  const void* cu;
  int64_t cu_stride;
  int32_t cu_is_64;
};

cudaError_t launch_update(int dtype, const UpdateArgs& a, int width, bool packet, dim3 grid, cudaStream_t s);
cudaError_t launch_varlen_states(int dtype, const VarlenArgs& a, bool packet, dim3 grid, cudaStream_t s);
// update_shift_kernel (kUpdateRows batch rows per thread)
cudaError_t launch_update_shift(int dtype, const UpdateArgs& a, int width, dim3 grid, cudaStream_t s);
// seqlen == 1 decode kernels; `kind` is one of kDecode*, the grid is derived from the args
cudaError_t launch_decode(int dtype, int kind, const UpdateArgs& a, int width, cudaStream_t s);
// channels one thread of a decode kernel covers (the host checks dim and alignment against it)
int decode_channels_per_thread(int kind, int dtype);

}  // namespace cc1d
