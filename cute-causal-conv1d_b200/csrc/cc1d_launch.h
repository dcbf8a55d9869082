// Host-side interface between the C-ABI launchers (cc1d_abi.cu) and the
// per-element-type kernel translation units.  Each kernel file is compiled once per
// element type with -DCC1D_DT=<cc1d_dtype>, which names its entry points
// <name>_f32 / <name>_f16 / <name>_bf16.
#pragma once

#include <cuda_runtime.h>

#include "cc1d_common.cuh"

namespace cc1d {

constexpr int kLayoutChannelLast = 0;  // stride over dim == 1
constexpr int kLayoutRows = 1;         // stride over seqlen == 1
constexpr int kLayoutStream = 2;       // channel-last, per-thread cp.async row stream
constexpr int kStreamDepth = 8;        // backward: rows in flight per thread (ring slots)
constexpr int kStreamDepthFwd = 16;    // forward: ring slots per thread (15 rows in flight)
constexpr int kStreamDepthEmit = 8;    // forward that writes varlen states: ring slots per thread
constexpr int kStreamThreads = 128;    // CTA size of the row-stream kernel
constexpr int kFwdStreamThreads = 512; // CTA size of the streamed forward (one CTA per SM)
#ifndef CC1D_FWD_PACKET
#define CC1D_FWD_PACKET 8
#endif
constexpr int kFwdPacketBytes = CC1D_FWD_PACKET;  // streamed forward: bytes of channels per lane and row
constexpr int kStreamDepthFwdSmall = 8;     // streamed forward of small problems: ring slots
constexpr int kFwdStreamThreadsSmall = 128; // streamed forward of small problems: CTA size
#ifndef CC1D_BWD_PACKET
#define CC1D_BWD_PACKET 8
#endif
#ifndef CC1D_BWD_THREADS
#define CC1D_BWD_THREADS 512
#endif
constexpr int kBwdPacketBytes = CC1D_BWD_PACKET;  // streamed backward: bytes of channels per lane and row
constexpr int kBwdStreamThreads = CC1D_BWD_THREADS;  // CTA size of the streamed backward (one CTA per SM at 128 registers)
constexpr int kLayoutRowStream = 3;    // (batch, dim, seqlen)-contiguous, per-lane sector stream
constexpr int kRowDepthBwd = 4;        // row-stream backward: ring slots (32-byte sectors) per lane and tensor
constexpr int kLayoutRowWalk = 4;      // (batch, dim, seqlen)-contiguous, lanes along the sequence
constexpr int kRowWalkDepth = 8;       // row walk: ring slots (16-byte packets) per lane and tensor
constexpr int kRowWalkThreads = 512;   // row walk: CTA size

struct LaunchShape {
  dim3 grid;
  int width;
  int layout;
  bool packet;  // 16-byte packets (alignment checked on the host) vs single elements
  bool silu;
  bool seq;
  bool emit;    // streamed forward only: also write the varlen states (ConvArgs::states)
  bool small;   // streamed forward only: the small-problem configuration (128-thread CTAs, 8-slot rings)
  size_t smem;
};

#define CC1D_DECLARE(name)                                                              \
  cudaError_t name##_f32(const ConvArgs&, const LaunchShape&, cudaStream_t);            \
  cudaError_t name##_f16(const ConvArgs&, const LaunchShape&, cudaStream_t);            \
  cudaError_t name##_bf16(const ConvArgs&, const LaunchShape&, cudaStream_t);           \
  const void* name##_kernel_ptr_f32(const LaunchShape&);                                \
  const void* name##_kernel_ptr_f16(const LaunchShape&);                                \
  const void* name##_kernel_ptr_bf16(const LaunchShape&);

CC1D_DECLARE(fwd)
CC1D_DECLARE(bwd)
#undef CC1D_DECLARE

// Launches `kernel` as a programmatic dependent launch: its CTAs may be scheduled while
// the previous kernel on the stream retires, and the kernel's first action,
// grid_dependency_wait(), holds them until that kernel has completed and its writes are
// visible.  Ordering with any earlier work is therefore the same as a plain launch.
template <typename Kernel, typename Arg>
inline cudaError_t launch_dependent(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                    const Arg& arg) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, arg);
}

// Sets the message returned by cc1d_last_error() on the calling thread.
void set_last_error(const char* msg);

cudaError_t rows_f32(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
cudaError_t rows_f16(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
cudaError_t rows_bf16(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
const void* rows_kernel_ptr_f32(bool bwd);
const void* rows_kernel_ptr_f16(bool bwd);
const void* rows_kernel_ptr_bf16(bool bwd);
cudaError_t rowwalk_f32(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
cudaError_t rowwalk_f16(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
cudaError_t rowwalk_bf16(bool bwd, const ConvArgs&, const LaunchShape&, cudaStream_t);
const void* rowwalk_kernel_ptr_f32(bool bwd, size_t smem);
const void* rowwalk_kernel_ptr_f16(bool bwd, size_t smem);
const void* rowwalk_kernel_ptr_bf16(bool bwd, size_t smem);

// Lets `kernel` use `bytes` of dynamic shared memory (above the 48 KB default) on the
// current device; the attribute is set once per kernel and device.
cudaError_t allow_dynamic_smem(const void* kernel, size_t bytes);

cudaError_t reduce_rows_f32(const ConvArgs&, int width, cudaStream_t);
cudaError_t reduce_rows_f16(const ConvArgs&, int width, cudaStream_t);
cudaError_t reduce_rows_bf16(const ConvArgs&, int width, cudaStream_t);

}  // namespace cc1d

#ifdef CC1D_DT
#if CC1D_DT == 0
#define CC1D_DT_TYPE float
#define CC1D_DT_SUFFIX f32
#elif CC1D_DT == 1
#define CC1D_DT_TYPE __half
#define CC1D_DT_SUFFIX f16
#else
#define CC1D_DT_TYPE __nv_bfloat16
#define CC1D_DT_SUFFIX bf16
#endif
#define CC1D_CAT2(a, b) a##_##b
#define CC1D_CAT(a, b) CC1D_CAT2(a, b)
#define CC1D_DT_NAME(name) CC1D_CAT(name, CC1D_DT_SUFFIX)
#endif
