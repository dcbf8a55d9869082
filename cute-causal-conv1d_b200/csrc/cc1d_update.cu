// Decode-time state update and varlen state gather (sm_100a).
//
// update: one thread per (batch row, VEC channels).  The output window is
// [state history | x]; outputs read the old state; the state is written after every
// output of the row is computed, by the same thread, so the in-place shift needs no
// synchronisation.  With channel-last x and state the VEC channels move as one 8-byte
// packet (256 contiguous bytes per warp); other layouts use VEC = 1 with the same code.
//
// varlen states: one thread per (sequence, state slot, VEC channels), a pure gather
// of the last state_len tokens of each packed sequence (zero where the sequence is
// shorter), bit exact.
#include "cc1d_common.cuh"
#include "cc1d_launch.h"
#include "cc1d_update_launch.h"

namespace cc1d {

template <typename T, int W, int VEC>
__global__ void __launch_bounds__(kThreads) update_kernel(const UpdateArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  // CTA tile: 32 channel packets x (8 warps x BR batch rows).  A thread owns one packet
  // for BR batch rows: it loads the weights once, issues the loads of all BR rows before
  // using any of them (the rows' memory latencies overlap), then computes and writes.
  // Positions inside a state row are 32-bit: the circular base cache % state_len is taken
  // once per row and every later position is one add and one wrap.
  constexpr int BR = kUpdateRows;
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int64_t nv = (a.dim + VEC - 1) / VEC;
  const int64_t nbx = (nv + 31) / 32;
  const int64_t cv = (blockIdx.x % nbx) * 32 + tx;
  const int64_t b0 = ((blockIdx.x / nbx) * 8 + ty) * BR;
  if (cv >= nv || b0 >= a.batch) return;
  const int64_t d0 = cv * VEC;
  const int T_len = static_cast<int>(a.seqlen);
  const int S = static_cast<int>(a.state_len);

  // phase 1: first inputs and row indices (independent loads, issued first).  A row
  // index that is negative or not below state_batch is a padding row; it is tested where
  // the row is used, so that no instruction waits on an index load before the others
  // are issued.
  int row[BR], base[BR];
  bool ok[BR];
  Packet<T, VEC> hist[BR][W - 1], x0[BR];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int64_t b = b0 + r;
    ok[r] = b < a.batch;
    if (ok[r]) x0[r] = ld_packet<T, VEC>(static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 * a.x.s1);
    row[r] = (ok[r] && a.indices) ? a.indices[b * a.indices_stride] : static_cast<int>(b);
    base[r] = (ok[r] && a.cache_seqlens) ? a.cache_seqlens[b * a.cache_stride] : 0;
  }

  auto live = [&](int r) { return static_cast<unsigned>(row[r]) < static_cast<unsigned>(a.state_batch); };
  float wv[W][VEC], bv[VEC];
  if (a.weight_vec) {  // contiguous fp32 (dim, W): this thread's VEC*W weights are adjacent
    const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(a.weight.data) + d0 * W);
    float flat[VEC * W];
#pragma unroll
    for (int q = 0; q < VEC * W / 4; ++q) {
      const float4 f = __ldg(wp + q);
      flat[4 * q] = f.x;
      flat[4 * q + 1] = f.y;
      flat[4 * q + 2] = f.z;
      flat[4 * q + 3] = f.w;
    }
#pragma unroll
    for (int v = 0; v < VEC; ++v)
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w][v] = flat[v * W + w];
  } else if (a.weight.dtype == CC1D_FLOAT32 && a.weight.s1 == 1) {
    const float* wp = static_cast<const float*>(a.weight.data);
#pragma unroll
    for (int v = 0; v < VEC; ++v)
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w][v] = d0 + v < a.dim ? __ldg(wp + (d0 + v) * a.weight.s0 + w) : 0.f;
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v)
#pragma unroll
      for (int w = 0; w < W; ++w)
        wv[w][v] = load_any(a.weight.data, a.weight.dtype, (d0 + v) * a.weight.s0 + w * a.weight.s1);
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) bv[v] = a.bias.data ? load_any(a.bias.data, a.bias.dtype, (d0 + v) * a.bias.s0) : 0.f;

  // history windows (circular: positions base-(W-1) .. base-1 mod S; otherwise the last
  // W-1 entries of the row)
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if (!ok[r] || !live(r)) continue;
    if (a.cache_seqlens) {
      base[r] %= S;
      if (base[r] < 0) base[r] += S;
    }
    const T* sp = static_cast<const T*>(a.state.data) + (int64_t)row[r] * a.state.s0 + d0 * a.state.s1;
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
      int pos = S - (W - 1) + i;
      if (a.cache_seqlens) {
        pos = base[r] - (W - 1) + i;  // >= -(W-1) >= -S
        if (pos < 0) pos += S;
      }
      hist[r][i] = ld_packet<T, VEC>(sp + (int64_t)pos * a.state.s2);
    }
  }

  // phase 2: outputs (the window is [history | x]; outputs use the old state)
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if (!ok[r]) continue;
    const int64_t b = b0 + r;
    const T* xp = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 * a.x.s1;
    T* op = static_cast<T*>(a.out.data) + b * a.out.s0 + d0 * a.out.s1;
    if (!live(r)) {  // padded batch row: zero output, state untouched
      float z[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) z[v] = 0.f;
      for (int t = 0; t < T_len; ++t) st_packet<T, VEC>(op + t * a.out.s2, pack<T, VEC>(z));
      continue;
    }
    float hw[W - 1][VEC];
#pragma unroll
    for (int i = 0; i < W - 1; ++i) unpack<T, VEC>(hist[r][i], hw[i]);
    for (int t = 0; t < T_len; ++t) {
      float xc[VEC];
      unpack<T, VEC>(t == 0 ? x0[r] : ld_packet<T, VEC>(xp + t * a.x.s2), xc);
      float acc[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float s = bv[v];
#pragma unroll
        for (int w = 0; w < W - 1; ++w) s = fmaf(wv[w][v], hw[w][v], s);
        s = fmaf(wv[W - 1][v], xc[v], s);
        if (a.silu) s = silu_fwd<T>(s);
        acc[v] = s;
      }
      st_packet<T, VEC>(op + t * a.out.s2, pack<T, VEC>(acc));
#pragma unroll
      for (int k = 0; k < W - 2; ++k)
#pragma unroll
        for (int v = 0; v < VEC; ++v) hw[k][v] = hw[k + 1][v];
#pragma unroll
      for (int v = 0; v < VEC; ++v) hw[W - 2][v] = xc[v];
    }
  }

  // phase 3: state writes (raw copies, bit exact)
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if (!ok[r] || !live(r)) continue;
    const T* xp = static_cast<const T*>(a.x.data) + (b0 + r) * a.x.s0 + d0 * a.x.s1;
    T* sp = static_cast<T*>(a.state.data) + (int64_t)row[r] * a.state.s0 + d0 * a.state.s1;
    if (a.cache_seqlens) {
      int pos = base[r];
      for (int t = 0; t < T_len; ++t) {  // in order: with seqlen > state_len the last write wins
        st_packet<T, VEC>(sp + (int64_t)pos * a.state.s2, t == 0 ? x0[r] : ld_packet<T, VEC>(xp + t * a.x.s2));
        pos = pos + 1 == S ? 0 : pos + 1;
      }
    } else if (S == W - 1 && T_len == 1) {
      // the whole old state is the history window: shift it from registers
#pragma unroll
      for (int i = 0; i + 1 < W - 1; ++i) st_packet<T, VEC>(sp + i * a.state.s2, hist[r][i + 1]);
      st_packet<T, VEC>(sp + (S - 1) * a.state.s2, x0[r]);
    } else {
      // new[s] = old[s + T] (s + T < S) or x[s + T - S].  Positions move down, so a group
      // of G positions is read completely before it is written, in ascending groups.
      constexpr int G = 4;
      for (int s0 = 0; s0 < S; s0 += G) {
        Packet<T, VEC> v[G];
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const int src = s0 + q + T_len;
          if (s0 + q < S)
            v[q] = (src < S) ? ld_packet<T, VEC>(sp + (int64_t)src * a.state.s2) : ld_packet<T, VEC>(xp + (int64_t)(src - S) * a.x.s2);
        }
#pragma unroll
        for (int q = 0; q < G; ++q)
          if (s0 + q < S) st_packet<T, VEC>(sp + (int64_t)(s0 + q) * a.state.s2, v[q]);
      }
    }
  }
}

// Shift update of a (batch, dim, state_len) state stored with its state_len entries per
// channel contiguous (stride 1) and channels state_len apart, for state_len == W-1 and
// no circular buffer.  The states of CH consecutive channels (8 bytes of x) are then one
// contiguous block of W-1 8-byte vectors, so a thread moves its channels' history with
// W-1 vector loads and stores instead of per-element accesses, and a warp covers 32
// consecutive blocks.  A thread takes BR batch rows and issues the
// loads of all of them (x, row index, state block) before using any.  The new state is
// assembled from the raw input elements (bit exact).
template <typename T, int W, int BR>
__global__ void __launch_bounds__(kThreads) update_shift_kernel(const UpdateArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  constexpr int CH = 8 / sizeof(T);  // channels per thread
  constexpr int S = W - 1;            // state entries per channel
  using Pk = Packet<T, CH>;
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int64_t nv = a.dim / CH;
  const int64_t nbx = (nv + 31) / 32;
  const int64_t cv = (blockIdx.x % nbx) * 32 + tx;
  const int64_t b0 = ((blockIdx.x / nbx) * (kThreads / 32) + ty) * BR;
  if (cv >= nv || b0 >= a.batch) return;
  const int64_t d0 = cv * CH;
  const int T_len = static_cast<int>(a.seqlen);

  int row[BR];
  bool ok[BR];
  Pk x0[BR], blk[BR][S];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int64_t b = b0 + r;
    ok[r] = b < a.batch;
    if (ok[r]) x0[r] = ld_packet<T, CH>(static_cast<const T*>(a.x.data) + b * a.x.s0 + d0);
    row[r] = (ok[r] && a.indices) ? a.indices[b * a.indices_stride] : static_cast<int>(b);
    if (row[r] >= a.state_batch) row[r] = -1;  // out of range: a padding row, nothing written
  }
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if (!ok[r] || row[r] < 0) continue;
    const T* sp = static_cast<const T*>(a.state.data) + (int64_t)row[r] * a.state.s0 + d0 * S;
#pragma unroll
    for (int q = 0; q < S; ++q) blk[r][q] = ld_packet<T, CH>(sp + q * CH);
  }

  float wv[W][CH], bv[CH];
  if (a.weight_vec) {  // contiguous fp32 (dim, W): this thread's CH*W weights are adjacent
    const float2* wp = reinterpret_cast<const float2*>(static_cast<const float*>(a.weight.data) + d0 * W);
#pragma unroll
    for (int q = 0; q < CH * W / 2; ++q) {
      const float2 f = __ldg(wp + q);
      wv[(2 * q) % W][(2 * q) / W] = f.x;
      wv[(2 * q + 1) % W][(2 * q + 1) / W] = f.y;
    }
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int w = 0; w < W; ++w)
        wv[w][c] = load_any(a.weight.data, a.weight.dtype, (d0 + c) * a.weight.s0 + w * a.weight.s1);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) bv[c] = a.bias.data ? load_any(a.bias.data, a.bias.dtype, (d0 + c) * a.bias.s0) : 0.f;

#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if (!ok[r]) continue;
    const int64_t b = b0 + r;
    const T* xp = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0;
    T* op = static_cast<T*>(a.out.data) + b * a.out.s0 + d0;
    if (row[r] < 0) {  // padded batch row: zero output, state untouched
      float z[CH];
#pragma unroll
      for (int c = 0; c < CH; ++c) z[c] = 0.f;
      for (int t = 0; t < T_len; ++t) st_packet<T, CH>(op + t * a.out.s2, pack<T, CH>(z));
      continue;
    }
    // the history of channel c is elements c*S .. c*S+S-1 of the block
    T hr[S][CH];
#pragma unroll
    for (int e = 0; e < S * CH; ++e) hr[e % S][e / S] = blk[r][e / CH].v[e % CH];
    for (int t = 0; t < T_len; ++t) {
      const Pk xr = t == 0 ? x0[r] : ld_packet<T, CH>(xp + t * a.x.s2);
      float acc[CH];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float s = bv[c];
#pragma unroll
        for (int w = 0; w < S; ++w) s = fmaf(wv[w][c], to_f32(hr[w][c]), s);
        s = fmaf(wv[W - 1][c], to_f32(xr.v[c]), s);
        if (a.silu) s = silu_fwd<T>(s);
        acc[c] = s;
      }
      st_packet<T, CH>(op + t * a.out.s2, pack<T, CH>(acc));
#pragma unroll
      for (int c = 0; c < CH; ++c) {
#pragma unroll
        for (int k = 0; k + 1 < S; ++k) hr[k][c] = hr[k + 1][c];
        hr[S - 1][c] = xr.v[c];
      }
    }
    // the new state: the last S entries of [old | x], back in block order
    Pk nb[S];
#pragma unroll
    for (int e = 0; e < S * CH; ++e) nb[e / CH].v[e % CH] = hr[e % S][e / S];
    T* sp = static_cast<T*>(a.state.data) + (int64_t)row[r] * a.state.s0 + d0 * S;
#pragma unroll
    for (int q = 0; q < S; ++q) st_packet<T, CH>(sp + q * CH, nb[q]);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) varlen_states_kernel(const VarlenArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  const int64_t nv = (a.dim + VEC - 1) / VEC;
  const int64_t total = nv * a.state_len * a.batch;
  for (int64_t item = (int64_t)blockIdx.x * kThreads + threadIdx.x; item < total;
       item += (int64_t)gridDim.x * kThreads) {
    const int64_t cv = item % nv;
    int64_t r = item / nv;
    const int64_t s = r % a.state_len;
    const int64_t b = r / a.state_len;
    const int64_t begin = a.cu_is_64 ? static_cast<const int64_t*>(a.cu)[b * a.cu_stride]
                                     : static_cast<const int32_t*>(a.cu)[b * a.cu_stride];
    const int64_t end = a.cu_is_64 ? static_cast<const int64_t*>(a.cu)[(b + 1) * a.cu_stride]
                                   : static_cast<const int32_t*>(a.cu)[(b + 1) * a.cu_stride];
    const int64_t token = end - a.state_len + s;
    T* dst = static_cast<T*>(a.states.data) + b * a.states.s0 + cv * VEC * a.states.s1 + s * a.states.s2;
    Packet<T, VEC> v;
    if (token >= begin && token < a.total_tokens) {  // rows past the end of x give zeros
      v = ld_packet<T, VEC>(static_cast<const T*>(a.x.data) + token * a.x.s0 + cv * VEC * a.x.s1);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) v.v[i] = from_f32<T>(0.f);
    }
    st_packet<T, VEC>(dst, v);
  }
}

template <typename T>
static cudaError_t launch_update_t(const UpdateArgs& a, int width, bool packet, dim3 grid, cudaStream_t s) {
  constexpr int PV = 8 / sizeof(T);  // 8-byte packets: more threads, fewer registers per thread
  cudaError_t e;
  switch (width * 2 + (packet ? 1 : 0)) {
    case 4: e = launch_dependent(update_kernel<T, 2, 1>, grid, dim3(kThreads), 0, s, a); break;
    case 5: e = launch_dependent(update_kernel<T, 2, PV>, grid, dim3(kThreads), 0, s, a); break;
    case 6: e = launch_dependent(update_kernel<T, 3, 1>, grid, dim3(kThreads), 0, s, a); break;
    case 7: e = launch_dependent(update_kernel<T, 3, PV>, grid, dim3(kThreads), 0, s, a); break;
    case 8: e = launch_dependent(update_kernel<T, 4, 1>, grid, dim3(kThreads), 0, s, a); break;
    case 9: e = launch_dependent(update_kernel<T, 4, PV>, grid, dim3(kThreads), 0, s, a); break;
    default: return cudaErrorInvalidValue;
  }
  return e;
}

template <typename T>
static cudaError_t launch_varlen_t(const VarlenArgs& a, bool packet, dim3 grid, cudaStream_t s) {
  constexpr int PV = 16 / sizeof(T);
  const cudaError_t e = packet ? launch_dependent(varlen_states_kernel<T, PV>, grid, dim3(kThreads), 0, s, a)
                               : launch_dependent(varlen_states_kernel<T, 1>, grid, dim3(kThreads), 0, s, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_update(int dtype, const UpdateArgs& a, int width, bool packet, dim3 grid, cudaStream_t s) {
  switch (dtype) {
    case CC1D_FLOAT32: return launch_update_t<float>(a, width, packet, grid, s);
    case CC1D_FLOAT16: return launch_update_t<__half>(a, width, packet, grid, s);
    case CC1D_BFLOAT16: return launch_update_t<__nv_bfloat16>(a, width, packet, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_shift_t(const UpdateArgs& a, int width, dim3 grid, cudaStream_t s) {
  constexpr int BR = kUpdateRows;
  switch (width) {
    case 2: return launch_dependent(update_shift_kernel<T, 2, BR>, grid, dim3(kThreads), 0, s, a);
    case 3: return launch_dependent(update_shift_kernel<T, 3, BR>, grid, dim3(kThreads), 0, s, a);
    case 4: return launch_dependent(update_shift_kernel<T, 4, BR>, grid, dim3(kThreads), 0, s, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_update_shift(int dtype, const UpdateArgs& a, int width, dim3 grid, cudaStream_t s) {
  switch (dtype) {
    case CC1D_FLOAT32: return launch_shift_t<float>(a, width, grid, s);
    case CC1D_FLOAT16: return launch_shift_t<__half>(a, width, grid, s);
    case CC1D_BFLOAT16: return launch_shift_t<__nv_bfloat16>(a, width, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_varlen_states(int dtype, const VarlenArgs& a, bool packet, dim3 grid, cudaStream_t s) {
  switch (dtype) {
    case CC1D_FLOAT32: return launch_varlen_t<float>(a, packet, grid, s);
    case CC1D_FLOAT16: return launch_varlen_t<__half>(a, packet, grid, s);
    case CC1D_BFLOAT16: return launch_varlen_t<__nv_bfloat16>(a, packet, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cc1d
