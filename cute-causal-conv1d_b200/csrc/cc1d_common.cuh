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
// A packet is VEC consecutive elements; 4-, 8- and 16-byte packets move as one
// access (the caller guarantees the alignment), others element by element.
template <typename T, int VEC> struct alignas(sizeof(T) * VEC) Packet { T v[VEC]; };

template <typename T, int VEC>
__device__ __forceinline__ Packet<T, VEC> ld_packet(const T* p) {
  Packet<T, VEC> r;
  if constexpr (sizeof(T) * VEC == 16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    r = *reinterpret_cast<Packet<T, VEC>*>(&u);
  } else if constexpr (sizeof(T) * VEC == 8) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    r = *reinterpret_cast<Packet<T, VEC>*>(&u);
  } else if constexpr (sizeof(T) * VEC == 4) {
    unsigned u = __ldg(reinterpret_cast<const unsigned*>(p));
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
  } else if constexpr (sizeof(T) * VEC == 8) {
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(&r);
  } else if constexpr (sizeof(T) * VEC == 4) {
    *reinterpret_cast<unsigned*>(p) = *reinterpret_cast<const unsigned*>(&r);
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

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel on its stream is still running;
// this wait returns once that kernel has completed and its writes are visible.  For a
// kernel launched without the attribute it returns at once.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------ SiLU
// Hardware approximations (PTX): 2^v and 1/v, flushing subnormals to zero.
__device__ __forceinline__ float ex2_approx(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float tanh_approx(float v) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// exp(-p) = 2^(-p * log2(e)), clamped to 1e30 so that 1 + e and e * sigmoid stay finite
// for very negative p (sigmoid(p) is then 1e-30, i.e. 0 to working precision).
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float exp_neg(float p) { return fminf(ex2_approx(-kLog2e * p), 1e30f); }

// Forward SiLU.  16-bit outputs use the single-MUFU identity
// silu(p) = h * tanh(h) + h with h = p / 2 (sigmoid(p) = (1 + tanh(p/2)) / 2); its
// approximation error is far below the tolerance of a 16-bit result.  fp32 outputs use
// p * sigmoid(p) with sigmoid(p) = 1 / (1 + exp(-p)).
template <typename T>
__device__ __forceinline__ float silu_fwd(float p) {
  if constexpr (std::is_same<T, float>::value) {
    return p * rcp_approx(1.0f + exp_neg(p));
  } else {
    float h = 0.5f * p;
    return fmaf(h, tanh_approx(h), h);
  }
}

// d silu(p) / dp = s * (1 + p * (1 - s)) with s = sigmoid(p); 1 - s = e * s with
// e = exp(-p), which has no cancellation for large p.
__device__ __forceinline__ float silu_grad(float p) {
  const float e = exp_neg(p);
  const float s = rcp_approx(1.0f + e);
  return s * fmaf(p, e * s, 1.0f);
}

// ------------------------------------------------------------ fp32x2 arithmetic
// sm_100 executes fp32 FMA / MUL / ADD on register pairs in one instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// Packet <-> fp32 pairs.  A bf16 is the upper half of an fp32, so a bf16 pair widens
// with one shift and one mask.
template <typename T, int VEC>
__device__ __forceinline__ void unpack2(const Packet<T, VEC>& r, float2 (&f)[VEC / 2]) {
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) {
    if constexpr (std::is_same<T, float>::value) {
      f[i] = make_float2(r.v[2 * i], r.v[2 * i + 1]);
    } else if constexpr (std::is_same<T, __half>::value) {
      f[i] = __half22float2(*reinterpret_cast<const __half2*>(&r.v[2 * i]));
    } else {
      const unsigned u = *reinterpret_cast<const unsigned*>(&r.v[2 * i]);
      f[i] = make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    }
  }
}
template <typename T, int VEC>
__device__ __forceinline__ Packet<T, VEC> pack2(const float2 (&f)[VEC / 2]) {
  Packet<T, VEC> r;
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) {
    if constexpr (std::is_same<T, float>::value) {
      r.v[2 * i] = f[i].x;
      r.v[2 * i + 1] = f[i].y;
    } else if constexpr (std::is_same<T, __half>::value) {
      *reinterpret_cast<__half2*>(&r.v[2 * i]) = __floats2half2_rn(f[i].x, f[i].y);
    } else {
      *reinterpret_cast<__nv_bfloat162*>(&r.v[2 * i]) = __floats2bfloat162_rn(f[i].x, f[i].y);
    }
  }
  return r;
}

// SiLU of a pair whose argument was pre-scaled by 1/2 (h = p/2), 16-bit outputs:
// silu(p) = h * tanh(h) + h.
__device__ __forceinline__ float2 silu_half_arg2(float2 h) {
  return ffma2(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h);
}
__device__ __forceinline__ float2 exp_neg2(float2 p) {
  const float2 v = fmul2(make_float2(-kLog2e, -kLog2e), p);
  return make_float2(fminf(ex2_approx(v.x), 1e30f), fminf(ex2_approx(v.y), 1e30f));
}
__device__ __forceinline__ float2 silu_exact2(float2 p) {
  const float2 d = fadd2(make_float2(1.0f, 1.0f), exp_neg2(p));
  return fmul2(p, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}
// d silu / dp of a pair (see silu_grad).
__device__ __forceinline__ float2 silu_grad2(float2 p) {
  const float2 e = exp_neg2(p);
  const float2 d = fadd2(make_float2(1.0f, 1.0f), e);
  const float2 s = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  return fmul2(s, ffma2(p, fmul2(e, s), make_float2(1.0f, 1.0f)));
}

// Twice d silu / dp of a pair whose argument was pre-scaled by 1/2 (h = p/2), one MUFU
// per element: with t = tanh(h), sigmoid(p) = (1 + t)/2 and
//   silu'(p) = sigmoid(p) * (1 + p * (1 - sigmoid(p))) = (1 + t) * (1 + h * (1 - t)) / 2.
// Used for 16-bit tensors, whose outputs tolerate tanh.approx's error.
__device__ __forceinline__ float2 silu_grad_half_arg2_x2(float2 h) {
  const float2 t = make_float2(tanh_approx(h.x), tanh_approx(h.y));
  const float2 one = make_float2(1.0f, 1.0f);
  const float2 omt = ffma2(t, make_float2(-1.0f, -1.0f), one);  // 1 - t
  return fmul2(fadd2(one, t), ffma2(h, omt, one));
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
  // streamed kernels: work is split into warp units.  A warp column is 32 consecutive
  // channel packets (packet block pb) of one batch row b, numbered col = pb * batch + b;
  // columns < seg_r are cut into seg_q + 1 sequence segments, the others into seg_q;
  // unit u is one (column, segment).  The units of one packet block are contiguous.
  int64_t ncol, seg_q, seg_r, units;
  // forward of packed sequences that also writes their varlen states (batch == 1):
  // states (nseq, dim, state_len) in x's dtype, cu_seqlens (nseq + 1,) int32 or int64
  TensorArg states;
  const void* cu;
  int64_t cu_stride;
  int cu_is_64, nseq, state_len;
};

// First warp unit of column c (c == ncol gives the total).
__host__ __device__ inline int64_t first_unit(const ConvArgs& a, int64_t c) {
  return c < a.seg_r ? c * (a.seg_q + 1) : a.seg_r * (a.seg_q + 1) + (c - a.seg_r) * a.seg_q;
}

// The (column, segment) of warp unit u, the column's segment count and its first unit.
// 32-bit arithmetic: the planners keep units, columns and seqlen below 2^31.
struct WarpUnit {
  int64_t col, seg, nseg, first;
};
__device__ __forceinline__ WarpUnit warp_unit(const ConvArgs& a, int64_t unit) {
  WarpUnit w;
  const unsigned u = static_cast<unsigned>(unit);
  const unsigned q = static_cast<unsigned>(a.seg_q), q1 = q + 1u;
  const unsigned big = static_cast<unsigned>(a.seg_r) * q1;
  if (u < big) {
    const unsigned c = u / q1;
    w.col = c;
    w.seg = u - c * q1;
    w.nseg = q1;
    w.first = c * q1;
  } else {
    const unsigned v = u - big;
    const unsigned c = v / q;
    w.col = a.seg_r + c;
    w.seg = v - c * q;
    w.nseg = q;
    w.first = big + c * q;
  }
  return w;
}

// Start of part s when len items are cut into n parts whose lengths differ by at most
// one (the first len % n parts are one longer); s == n gives len.  32-bit arithmetic.
__device__ __forceinline__ int64_t part_start(int64_t s, int64_t n, int64_t len) {
  const unsigned un = static_cast<unsigned>(n), ul = static_cast<unsigned>(len), us = static_cast<unsigned>(s);
  const unsigned base = ul / un, rem = ul - base * un;
  return static_cast<int64_t>(us * base + min(us, rem));
}

// seq_idx of consecutive rows for a warp's walk: 32 rows at a time are fetched with one
// coalesced load (lane i holds row block + i), one block ahead of use, and each row's
// value reaches every lane by __shfl_sync - no per-row dependent load.  Rows at or past
// `end` read as -1.  Every lane of the warp must call next() together.
struct SeqFeed {
  const int* p;
  int64_t stride, pos, end;  // pos: first row of the next block to load
  int cur, nxt, k;
  __device__ __forceinline__ int load(int lane) const {
    const int64_t r = pos + lane;
    return r < end ? __ldg(p + r * stride) : -1;
  }
  __device__ __forceinline__ void start(const int* row0, int64_t s, int64_t first, int64_t end_rows, int lane) {
    p = row0;
    stride = s;
    end = end_rows;
    pos = first;
    cur = load(lane);
    pos += 32;
    nxt = load(lane);
    pos += 32;
    k = 0;
  }
  __device__ __forceinline__ int next(int lane) {
    const int v = __shfl_sync(0xffffffffu, cur, k);
    if (++k == 32) {
      k = 0;
      cur = nxt;
      nxt = load(lane);
      pos += 32;
    }
    return v;
  }
  // Whether the next n rows (n divides 32, k a multiple of n) all carry the value v.
  __device__ __forceinline__ bool next_all(int lane, int n, int v) const {
    return __all_sync(0xffffffffu, static_cast<unsigned>(lane - k) >= static_cast<unsigned>(n) || cur == v);
  }
  // Passes over the next n rows (n divides 32, k a multiple of n).
  __device__ __forceinline__ void skip(int lane, int n) {
    k += n;
    if (k == 32) {
      k = 0;
      cur = nxt;
      nxt = load(lane);
      pos += 32;
    }
  }
};

// Weight and bias of VEC consecutive channels, as fp32.
// fp32 (dim, W) weight with unit channel stride and fp32 unit-stride bias (or none) take
// a branch-free path whose loads all issue back to back.
template <int W, int VEC>
__device__ __forceinline__ void load_params(const ConvArgs& a, int64_t d0, float (&wv)[W][VEC],
                                            float (&bv)[VEC]) {
  const bool fast = d0 + VEC <= a.dim && a.weight.dtype == CC1D_FLOAT32 && a.weight.s1 == 1 &&
                    (!a.bias.data || (a.bias.dtype == CC1D_FLOAT32 && a.bias.s0 == 1));
  if (fast) {
    const float* wp = static_cast<const float*>(a.weight.data) + d0 * a.weight.s0;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w][v] = __ldg(wp + v * a.weight.s0 + w);
    }
    if (a.bias.data) {
      const float* bp = static_cast<const float*>(a.bias.data) + d0;
#pragma unroll
      for (int v = 0; v < VEC; ++v) bv[v] = __ldg(bp + v);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) bv[v] = 0.f;
    }
    return;
  }
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

// x at the W-1 rows before position l0 of one lane's VEC channels d0.. (rows before 0
// come from initial_states, or are zero).  Away from position 0 all loads are issued
// before any value is used.
template <typename T, int W, int VEC>
__device__ __forceinline__ void load_window(const ConvArgs& a, int64_t b, int64_t d0, int64_t l0,
                                            float2 (&xw)[W - 1][VEC / 2]) {
  constexpr int H = VEC / 2;
  const T* col = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0;
  if (l0 >= W - 1) {
    Packet<T, VEC> raw[W - 1];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) raw[k] = ld_packet<T, VEC>(col + (l0 - (W - 1) + k) * a.x.s2);
#pragma unroll
    for (int k = 0; k < W - 1; ++k) unpack2<T, VEC>(raw[k], xw[k]);
    return;
  }
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    const int64_t l = l0 - (W - 1) + k;
    if (l >= 0) {
      unpack2<T, VEC>(ld_packet<T, VEC>(col + l * a.x.s2), xw[k]);
    } else if (a.init.data) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const int64_t o = b * a.init.s0 + (d0 + 2 * i) * a.init.s1 + (W - 1 + l) * a.init.s2;
        xw[k][i] = make_float2(load_any(a.init.data, a.init.dtype, o), load_any(a.init.data, a.init.dtype, o + a.init.s1));
      }
    } else {
#pragma unroll
      for (int i = 0; i < H; ++i) xw[k][i] = make_float2(0.f, 0.f);
    }
  }
}

}  // namespace cc1d
