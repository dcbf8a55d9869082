// Shared device helpers for the causal_conv1d sm_100a kernels.
//
// Element types, 16-byte vector loads/stores, fp32 conversions, SiLU and its
// derivative, and the plain-old-data argument blocks the launchers pass by value.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "causal_conv1d_b200.h"

namespace cc1d {

constexpr int kThreads = 256;  // every kernel launches 256-thread CTAs

// ------------------------------------------------------------------ element types
template <int DT> struct DTypeOf;
template <> struct DTypeOf<CC1D_FLOAT32> { using type = float; };
template <> struct DTypeOf<CC1D_FLOAT16> { using type = __half; };
template <> struct DTypeOf<CC1D_BFLOAT16> { using type = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Scalar access to tensors whose dtype is only known at run time (parameters and
// states, read once per thread).
__device__ __forceinline__ float load_any(const void* p, int dt, int64_t i) {
  if (dt == CC1D_FLOAT32) return static_cast<const float*>(p)[i];
  if (dt == CC1D_FLOAT16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void store_any(void* p, int dt, int64_t i, float v) {
  if (dt == CC1D_FLOAT32) static_cast<float*>(p)[i] = v;
  else if (dt == CC1D_FLOAT16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// ------------------------------------------------------------ VEC-element packets
// A packet is VEC consecutive elements; for VEC*sizeof(T) == 16 it moves as one
// 128-bit access, otherwise element by element.
template <typename T, int VEC> struct alignas(sizeof(T) * VEC) Packet { T v[VEC]; };

template <typename T, int VEC>
__device__ __forceinline__ Packet<T, VEC> ld_packet(const T* p) {
  Packet<T, VEC> r;
  if constexpr (sizeof(T) * VEC == 16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    r = *reinterpret_cast<Packet<T, VEC>*>(&u);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = p[i];
  }
  return r;
}

template <typename T, int VEC>
__device__ __forceinline__ void st_packet(T* p, const Packet<T, VEC>& r) {
  if constexpr (sizeof(T) * VEC == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(&r);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = r.v[i];
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void unpack(const Packet<T, VEC>& r, float (&f)[VEC]) {
  if constexpr (VEC % 2 == 0 && !std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      float2 t;
      if constexpr (std::is_same<T, __half>::value)
        t = __half22float2(*reinterpret_cast<const __half2*>(&r.v[i]));
      else
        t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.v[i]));
      f[i] = t.x;
      f[i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f32(r.v[i]);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ Packet<T, VEC> pack(const float (&f)[VEC]) {
  Packet<T, VEC> r;
  if constexpr (VEC % 2 == 0 && !std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      if constexpr (std::is_same<T, __half>::value)
        *reinterpret_cast<__half2*>(&r.v[i]) = __floats2half2_rn(f[i], f[i + 1]);
      else
        *reinterpret_cast<__nv_bfloat162*>(&r.v[i]) = __floats2bfloat162_rn(f[i], f[i + 1]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = from_f32<T>(f[i]);
  }
  return r;
}

// --------------------------------------------------------------- cp.async ring
// Asynchronous global->shared copy of one packet (Ampere-style LDGSTS, still the
// cheapest way on sm_100 for a thread to keep many small loads in flight without
// holding registers).  `valid == false` writes zeros and reads nothing.
template <int BYTES>
__device__ __forceinline__ void cp_async_packet(void* smem_dst, const void* gsrc, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  const int src_size = valid ? BYTES : 0;
  if constexpr (BYTES == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gsrc), "r"(src_size) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;\n" ::"r"(s), "l"(gsrc), "n"(BYTES), "r"(src_size)
                 : "memory");
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------ SiLU
// Forward SiLU.  16-bit outputs use the single-MUFU identity
// silu(p) = h * tanh(h) + h with h = p / 2 (sigmoid(p) = (1 + tanh(p/2)) / 2), whose
// approximation error sits far below one 16-bit ulp.  fp32 outputs use
// p / (1 + exp(-p)) with the fast exponential and a fast divide.
__device__ __forceinline__ float tanh_approx(float v) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

template <typename T>
__device__ __forceinline__ float silu_fwd(float p) {
  if constexpr (std::is_same<T, float>::value) {
    float e = fminf(__expf(-p), 1e30f);
    return __fdividef(p, 1.0f + e);
  } else {
    float h = 0.5f * p;
    return fmaf(h, tanh_approx(h), h);
  }
}

// d silu(p) / dp = s * (1 + p * (1 - s)) with s = sigmoid(p).  Written with
// e = exp(-p) so that 1 - s = e * s has no cancellation for large p; e is clamped
// so that e * s stays finite for very negative p.
__device__ __forceinline__ float silu_grad(float p) {
  float e = fminf(__expf(-p), 1e30f);
  float s = __fdividef(1.0f, 1.0f + e);
  return s * fmaf(p, e * s, 1.0f);
}

// ------------------------------------------------------------- argument blocks
struct TensorArg {
  void* data;
  int32_t dtype;
  int64_t s0, s1, s2;
};

__host__ __device__ inline TensorArg tensor_arg(const cc1d_tensor& t) {
  TensorArg a;
  a.data = t.data;
  a.dtype = t.dtype;
  a.s0 = t.stride[0];
  a.s1 = t.stride[1];
  a.s2 = t.stride[2];
  return a;
}

struct ConvArgs {
  int64_t batch, dim, seqlen;
  TensorArg x, weight, bias, seq_idx, init, final_states, out;  // forward
  TensorArg dout, dfinal, dx, dinit;                             // backward
  float* dweight;
  float* dbias;
  float* partials;          // [num_partials][dim][W+1] fp32, backward only
  unsigned int* counters;   // one arrival counter per channel tile, backward only
  // launch geometry (decided by the host)
  int tx_shift;             // channel-last: log2 of threads along channels per CTA
  int64_t nv;               // channel-last: channel packets; row kernels: unused
  int64_t chunk;            // sequence positions per thread (channel-last) / per group (row)
  int64_t nbx, nby;         // CTA grid factors (see each kernel)
  int g_shift;              // row kernels: log2 of lanes per row group
  int rounds;               // row kernels: rounds per chunk
  int64_t nck;              // row kernels: chunks per row
};

// Weight and bias of VEC consecutive channels, as fp32.
template <int W, int VEC>
__device__ __forceinline__ void load_params(const ConvArgs& a, int64_t d0, float (&wv)[W][VEC],
                                            float (&bv)[VEC]) {
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    const int64_t d = d0 + v;
    const bool ok = d < a.dim;
#pragma unroll
    for (int w = 0; w < W; ++w)
      wv[w][v] = ok ? load_any(a.weight.data, a.weight.dtype, d * a.weight.s0 + w * a.weight.s1) : 0.f;
    bv[v] = (ok && a.bias.data) ? load_any(a.bias.data, a.bias.dtype, d * a.bias.s0) : 0.f;
  }
}

}  // namespace cc1d
