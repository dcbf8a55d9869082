// Single-token decode update (seqlen == 1), the serving hot loop of the update op.
//
// A decode step moves a few bytes per channel (x, W-1 history entries, the state write,
// the output), so a launch of 10-20 MB is bound by how many bytes are in flight while
// the first DRAM round trip completes, not by instruction count.  These kernels give
// every thread one 16-byte packet of channels of BR batch rows, issue every global load
// of those rows (x, the row index and circular position, then the history) before any
// value is used, and size the grid so that the whole problem is resident at once:
//
//   decode_cl_kernel    conv_state with channels contiguous ((B, S, D) storage, the
//                       reference kernels' layout): W-1 history packets per row, one
//                       packet store (circular) or W-1 (shift).
//   decode_block_kernel conv_state (B, D, W-1) with the W-1 entries of a channel
//                       contiguous and no circular buffer: the histories of a packet's
//                       channels are one block of W-1 16-byte vectors, shifted in
//                       registers and written back whole.
//   decode_ring_kernel  conv_state (B, D, S) with the S entries of a channel contiguous,
//                       circular buffer, 16-bit types, S % 4 == 0: a channel's W-1
//                       history entries lie in at most two aligned 8-byte words of its
//                       row (the row's 32-byte sector is what DRAM moves either way), the
//                       new entry is one 2-byte store.
//
// All three keep the semantics of update_kernel: outputs use the old state, a row whose
// state index is negative or >= state_batch gets a zero output and no state write, the
// circular position is cache_seqlens[b] mod S (non-negative), state values are copied
// bit exact.  Rows are independent; two batch rows gathering the same state row race,
// as in the reference.
#include "cc1d_common.cuh"
#include "cc1d_launch.h"
#include "cc1d_update_launch.h"

// Launch shapes, measured on B200 at config 3 (B=128, D=8192, bf16, graphs of 16
// launches): decode_cl/block with 4 batch rows per thread (128 CTAs, every load of a
// thread issued together) took 5.2-6.2 us against 8.3-9.8 us with 1 row (512 CTAs, more
// than one wave) and 6.1-6.9 us with 2; decode_ring with 2 channels and 1 row per thread
// took 12.9-13.0 us against 18.7-22.6 us with 4 or 8 channels, and 13.0-18.1 us with 2 or
// 4 rows of 1 or 2 channels.
#ifndef CC1D_DECODE_ROWS
#define CC1D_DECODE_ROWS 4  // batch rows per thread (decode_cl_kernel, decode_block_kernel)
#endif
#ifndef CC1D_RING_ROWS
#define CC1D_RING_ROWS 1  // batch rows per thread (decode_ring_kernel)
#endif
#ifndef CC1D_RING_CH
#define CC1D_RING_CH 2  // channels per thread (decode_ring_kernel)
#endif
#ifndef CC1D_DECODE_THREADS
#define CC1D_DECODE_THREADS 256  // CTA size of the decode kernels (8 warps over batch rows)
#endif
#ifndef CC1D_DECODE_MINB
#define CC1D_DECODE_MINB 1  // resident CTAs per SM the register allocation must allow
#endif

namespace cc1d {

// Parameters of N consecutive channels starting at d0, fp32 in registers.
template <int W, int N>
__device__ __forceinline__ void decode_params(const UpdateArgs& a, int d0, float (&wv)[W][N], float (&bv)[N]) {
  if constexpr ((N * W) % 4 == 0) {
    if (a.weight_vec) {  // fp32 (dim, W) contiguous, 16-byte aligned: N*W adjacent floats
      const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(a.weight.data) + (int64_t)d0 * W);
      float flat[N * W];
#pragma unroll
      for (int q = 0; q < N * W / 4; ++q) {
        const float4 f = __ldg(wp + q);
        flat[4 * q] = f.x;
        flat[4 * q + 1] = f.y;
        flat[4 * q + 2] = f.z;
        flat[4 * q + 3] = f.w;
      }
#pragma unroll
      for (int v = 0; v < N; ++v)
#pragma unroll
        for (int w = 0; w < W; ++w) wv[w][v] = flat[v * W + w];
    } else {
#pragma unroll
      for (int v = 0; v < N; ++v)
#pragma unroll
        for (int w = 0; w < W; ++w)
          wv[w][v] = load_any(a.weight.data, a.weight.dtype, (int64_t)(d0 + v) * a.weight.s0 + w * a.weight.s1);
    }
  } else {
#pragma unroll
    for (int v = 0; v < N; ++v)
#pragma unroll
      for (int w = 0; w < W; ++w)
        wv[w][v] = load_any(a.weight.data, a.weight.dtype, (int64_t)(d0 + v) * a.weight.s0 + w * a.weight.s1);
  }
  if constexpr (N % 4 == 0) {
    if (a.bias_vec) {  // fp32 contiguous, 16-byte aligned
      const float4* bp = reinterpret_cast<const float4*>(static_cast<const float*>(a.bias.data) + d0);
#pragma unroll
      for (int q = 0; q < N / 4; ++q) {
        const float4 f = __ldg(bp + q);
        bv[4 * q] = f.x;
        bv[4 * q + 1] = f.y;
        bv[4 * q + 2] = f.z;
        bv[4 * q + 3] = f.w;
      }
      return;
    }
  }
#pragma unroll
  for (int v = 0; v < N; ++v) bv[v] = a.bias.data ? load_any(a.bias.data, a.bias.dtype, (int64_t)(d0 + v) * a.bias.s0) : 0.f;
}

// out = act(bias + sum_i w[i] * hist[i] + w[W-1] * x) for N channels.
template <typename T, int W, int N>
__device__ __forceinline__ void decode_out(const float (&wv)[W][N], const float (&bv)[N], const float (&h)[W - 1][N],
                                           const float (&xc)[N], bool silu, float (&acc)[N]) {
#pragma unroll
  for (int v = 0; v < N; ++v) {
    float s = bv[v];
#pragma unroll
    for (int i = 0; i < W - 1; ++i) s = fmaf(wv[i][v], h[i][v], s);
    s = fmaf(wv[W - 1][v], xc[v], s);
    acc[v] = silu ? silu_fwd<T>(s) : s;
  }
}

// Thread tile shared by the kernels: 32 lanes over consecutive channel groups of one
// batch row (a warp stays inside one row), the CTA's warps over groups of BR batch rows.
struct DecodeTile {
  int group;  // channel group index (groups of N channels)
  int b0;     // first batch row
  __device__ __forceinline__ DecodeTile(int ngroups, int rows_per_thread) {
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int nbx = (ngroups + 31) >> 5;
    group = (int)(blockIdx.x % (unsigned)nbx) * 32 + tx;
    b0 = ((int)(blockIdx.x / (unsigned)nbx) * (CC1D_DECODE_THREADS / 32) + ty) * rows_per_thread;
  }
};

__device__ __forceinline__ int wrap_mod(int v, int S) {
  v %= S;
  return v < 0 ? v + S : v;
}

template <typename T, int W, bool CIRC, int BR>
__global__ void __launch_bounds__(CC1D_DECODE_THREADS, CC1D_DECODE_MINB) decode_cl_kernel(const UpdateArgs a) {
  constexpr int V = 16 / sizeof(T);
  using Pk = Packet<T, V>;
  grid_dependency_wait();  // launched as a programmatic dependent launch
  const DecodeTile t((int)(a.dim / V), BR);
  if (t.group * V >= a.dim || t.b0 >= a.batch) return;
  const int d0 = t.group * V;
  const int S = (int)a.state_len;
  const T* xg = static_cast<const T*>(a.x.data);
  T* sg = static_cast<T*>(a.state.data);

  Pk x0[BR], hist[BR][W - 1];
  int row[BR], base[BR];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    const bool ok = b < a.batch;
    if (ok) x0[r] = ld_packet<T, V>(xg + (int64_t)b * a.x.s0 + d0);
    row[r] = !ok ? -1 : (a.indices ? a.indices[(int64_t)b * a.indices_stride] : b);
    base[r] = (CIRC && ok) ? a.cache_seqlens[(int64_t)b * a.cache_stride] : 0;
  }
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if ((unsigned)row[r] >= (unsigned)a.state_batch) continue;  // padding row, or past the batch
    if (CIRC) base[r] = wrap_mod(base[r], S);
    const T* sp = sg + (int64_t)row[r] * a.state.s0 + d0;
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
      int pos = i;  // shift update: the state is exactly the W-1 history entries
      if (CIRC) {
        pos = base[r] - (W - 1) + i;
        if (pos < 0) pos += S;
      }
      hist[r][i] = ld_packet<T, V>(sp + (int64_t)pos * a.state.s2);
    }
  }
  float wv[W][V], bv[V];
  decode_params<W, V>(a, d0, wv, bv);

#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    if (b >= a.batch) continue;
    T* op = static_cast<T*>(a.out.data) + (int64_t)b * a.out.s0 + d0;
    float acc[V];
    if ((unsigned)row[r] >= (unsigned)a.state_batch) {
#pragma unroll
      for (int v = 0; v < V; ++v) acc[v] = 0.f;
      st_packet<T, V>(op, pack<T, V>(acc));
      continue;
    }
    float h[W - 1][V], xc[V];
#pragma unroll
    for (int i = 0; i < W - 1; ++i) unpack<T, V>(hist[r][i], h[i]);
    unpack<T, V>(x0[r], xc);
    decode_out<T, W, V>(wv, bv, h, xc, a.silu != 0, acc);
    st_packet<T, V>(op, pack<T, V>(acc));
    T* sp = sg + (int64_t)row[r] * a.state.s0 + d0;
    if (CIRC) {
      st_packet<T, V>(sp + (int64_t)base[r] * a.state.s2, x0[r]);
    } else {
#pragma unroll
      for (int i = 0; i + 1 < W - 1; ++i) st_packet<T, V>(sp + (int64_t)i * a.state.s2, hist[r][i + 1]);
      st_packet<T, V>(sp + (int64_t)(W - 2) * a.state.s2, x0[r]);
    }
  }
}

template <typename T, int W, int BR>
__global__ void __launch_bounds__(CC1D_DECODE_THREADS, CC1D_DECODE_MINB) decode_block_kernel(const UpdateArgs a) {
  constexpr int CH = 16 / sizeof(T);  // channels per thread
  constexpr int S = W - 1;             // state entries per channel
  using Pk = Packet<T, CH>;
  grid_dependency_wait();  // launched as a programmatic dependent launch
  const DecodeTile t((int)(a.dim / CH), BR);
  if (t.group * CH >= a.dim || t.b0 >= a.batch) return;
  const int d0 = t.group * CH;
  const T* xg = static_cast<const T*>(a.x.data);
  T* sg = static_cast<T*>(a.state.data);

  Pk x0[BR], blk[BR][S];
  int row[BR];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    const bool ok = b < a.batch;
    if (ok) x0[r] = ld_packet<T, CH>(xg + (int64_t)b * a.x.s0 + d0);
    row[r] = !ok ? -1 : (a.indices ? a.indices[(int64_t)b * a.indices_stride] : b);
  }
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    if ((unsigned)row[r] >= (unsigned)a.state_batch) continue;
    const T* sp = sg + (int64_t)row[r] * a.state.s0 + (int64_t)d0 * S;
#pragma unroll
    for (int q = 0; q < S; ++q) blk[r][q] = ld_packet<T, CH>(sp + q * CH);
  }
  float wv[W][CH], bv[CH];
  decode_params<W, CH>(a, d0, wv, bv);

#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    if (b >= a.batch) continue;
    T* op = static_cast<T*>(a.out.data) + (int64_t)b * a.out.s0 + d0;
    float acc[CH];
    if ((unsigned)row[r] >= (unsigned)a.state_batch) {
#pragma unroll
      for (int c = 0; c < CH; ++c) acc[c] = 0.f;
      st_packet<T, CH>(op, pack<T, CH>(acc));
      continue;
    }
    // entry k of channel c is element c*S + k of the block
    float h[S][CH], xc[CH];
#pragma unroll
    for (int e = 0; e < S * CH; ++e) h[e % S][e / S] = to_f32(blk[r][e / CH].v[e % CH]);
    unpack<T, CH>(x0[r], xc);
    decode_out<T, W, CH>(wv, bv, h, xc, a.silu != 0, acc);
    st_packet<T, CH>(op, pack<T, CH>(acc));
    // the new state: entries 1..S-1 of the old one, then x (raw copies, bit exact)
    Pk nb[S];
#pragma unroll
    for (int e = 0; e < S * CH; ++e) {
      const int c = e / S, k = e % S;
      const int src = c * S + k + 1;
      nb[e / CH].v[e % CH] = (k + 1 < S) ? blk[r][src / CH].v[src % CH] : x0[r].v[c];
    }
    T* sp = sg + (int64_t)row[r] * a.state.s0 + (int64_t)d0 * S;
#pragma unroll
    for (int q = 0; q < S; ++q) st_packet<T, CH>(sp + q * CH, nb[q]);
  }
}

// The 16-bit element held in the low half of a 32-bit word.
template <typename T>
__device__ __forceinline__ T ring_elem(uint32_t r) {
  const unsigned short u = static_cast<unsigned short>(r & 0xffffu);
  return *reinterpret_cast<const T*>(&u);
}

template <typename T, int W, int CH, int BR>
__global__ void __launch_bounds__(CC1D_DECODE_THREADS, CC1D_DECODE_MINB) decode_ring_kernel(const UpdateArgs a) {
  static_assert(sizeof(T) == 2, "16-bit states only");
  using Pk = Packet<T, CH>;
  grid_dependency_wait();  // launched as a programmatic dependent launch
  const DecodeTile t((int)(a.dim / CH), BR);
  if (t.group * CH >= a.dim || t.b0 >= a.batch) return;
  const int d0 = t.group * CH;
  const int S = (int)a.state_len;  // a multiple of 4: a row is S/4 aligned 8-byte words
  const int nw = S >> 2;
  const T* xg = static_cast<const T*>(a.x.data);
  T* sg = static_cast<T*>(a.state.data);

  Pk x0[BR];
  int row[BR], base[BR];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    const bool ok = b < a.batch;
    if (ok) x0[r] = ld_packet<T, CH>(xg + (int64_t)b * a.x.s0 + d0);
    row[r] = !ok ? -1 : (a.indices ? a.indices[(int64_t)b * a.indices_stride] : b);
    base[r] = ok ? a.cache_seqlens[(int64_t)b * a.cache_stride] : 0;
  }
  // The history of a row starts at p0 = (base - (W-1)) mod S.  Entries p0 .. p0+W-2 (mod
  // S) lie in the 8-byte words k0 = p0/4 and (k0+1) mod S/4, at offsets o .. o+W-2 of
  // their concatenation, o = p0 % 4; the second word is needed only if o + W-2 >= 4.
  uint2 w0[BR][CH], w1[BR][CH];
  int off[BR];
#pragma unroll
  for (int r = 0; r < BR; ++r) {
    off[r] = 0;
    if ((unsigned)row[r] >= (unsigned)a.state_batch) continue;
    base[r] = wrap_mod(base[r], S);
    int p0 = base[r] - (W - 1);
    if (p0 < 0) p0 += S;
    const int k0 = p0 >> 2;
    const int k1 = k0 + 1 == nw ? 0 : k0 + 1;
    off[r] = p0 & 3;
    const bool two = off[r] + (W - 2) >= 4;  // the same for the whole warp (one batch row)
    const T* rp = sg + (int64_t)row[r] * a.state.s0 + (int64_t)d0 * S;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint2* wp = reinterpret_cast<const uint2*>(rp + (int64_t)c * S);
      w0[r][c] = __ldg(wp + k0);
      w1[r][c] = two ? __ldg(wp + k1) : make_uint2(0u, 0u);
    }
  }
  float wv[W][CH], bv[CH];
  decode_params<W, CH>(a, d0, wv, bv);

#pragma unroll
  for (int r = 0; r < BR; ++r) {
    const int b = t.b0 + r;
    if (b >= a.batch) continue;
    T* op = static_cast<T*>(a.out.data) + (int64_t)b * a.out.s0 + d0;
    float acc[CH];
    if ((unsigned)row[r] >= (unsigned)a.state_batch) {
#pragma unroll
      for (int c = 0; c < CH; ++c) acc[c] = 0.f;
      st_packet<T, CH>(op, pack<T, CH>(acc));
      continue;
    }
    const int j = off[r] >> 1;          // first 32-bit word holding entry o
    const int sh = (off[r] & 1) * 16;   // bit offset of entry o in it
    float h[W - 1][CH], xc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint32_t q0 = w0[r][c].x, q1 = w0[r][c].y, q2 = w1[r][c].x, q3 = w1[r][c].y;
      const uint32_t a0 = j ? q1 : q0, a1 = j ? q2 : q1, a2 = j ? q3 : q2;
      const uint32_t e01 = __funnelshift_r(a0, a1, sh);  // entries o, o+1
      const uint32_t e23 = __funnelshift_r(a1, a2, sh);  // entries o+2, o+3
      h[0][c] = to_f32(ring_elem<T>(e01));
      if constexpr (W > 2) h[1][c] = to_f32(ring_elem<T>(e01 >> 16));
      if constexpr (W > 3) h[2][c] = to_f32(ring_elem<T>(e23));
    }
    unpack<T, CH>(x0[r], xc);
    decode_out<T, W, CH>(wv, bv, h, xc, a.silu != 0, acc);
    st_packet<T, CH>(op, pack<T, CH>(acc));
    T* rp = sg + (int64_t)row[r] * a.state.s0 + (int64_t)d0 * S + base[r];
#pragma unroll
    for (int c = 0; c < CH; ++c) rp[(int64_t)c * S] = x0[r].v[c];
  }
}

template <typename T>
static cudaError_t launch_decode_t(int kind, const UpdateArgs& a, int width, dim3 grid, cudaStream_t s) {
  constexpr int BR = CC1D_DECODE_ROWS;
  const dim3 blk(CC1D_DECODE_THREADS);
  switch (kind * 8 + width) {
    case kDecodeClShift * 8 + 2: return launch_dependent(decode_cl_kernel<T, 2, false, BR>, grid, blk, 0, s, a);
    case kDecodeClShift * 8 + 3: return launch_dependent(decode_cl_kernel<T, 3, false, BR>, grid, blk, 0, s, a);
    case kDecodeClShift * 8 + 4: return launch_dependent(decode_cl_kernel<T, 4, false, BR>, grid, blk, 0, s, a);
    case kDecodeClCirc * 8 + 2: return launch_dependent(decode_cl_kernel<T, 2, true, BR>, grid, blk, 0, s, a);
    case kDecodeClCirc * 8 + 3: return launch_dependent(decode_cl_kernel<T, 3, true, BR>, grid, blk, 0, s, a);
    case kDecodeClCirc * 8 + 4: return launch_dependent(decode_cl_kernel<T, 4, true, BR>, grid, blk, 0, s, a);
    case kDecodeBlock * 8 + 2: return launch_dependent(decode_block_kernel<T, 2, BR>, grid, blk, 0, s, a);
    case kDecodeBlock * 8 + 3: return launch_dependent(decode_block_kernel<T, 3, BR>, grid, blk, 0, s, a);
    case kDecodeBlock * 8 + 4: return launch_dependent(decode_block_kernel<T, 4, BR>, grid, blk, 0, s, a);
    default: break;
  }
  if constexpr (sizeof(T) == 2) {
    constexpr int CH = CC1D_RING_CH, RR = CC1D_RING_ROWS;
    switch (kind * 8 + width) {
      case kDecodeRing * 8 + 2: return launch_dependent(decode_ring_kernel<T, 2, CH, RR>, grid, blk, 0, s, a);
      case kDecodeRing * 8 + 3: return launch_dependent(decode_ring_kernel<T, 3, CH, RR>, grid, blk, 0, s, a);
      case kDecodeRing * 8 + 4: return launch_dependent(decode_ring_kernel<T, 4, CH, RR>, grid, blk, 0, s, a);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

int decode_channels_per_thread(int kind, int dtype) {
  const int es = dtype == CC1D_FLOAT32 ? 4 : 2;
  return kind == kDecodeRing ? CC1D_RING_CH : 16 / es;
}

cudaError_t launch_decode(int dtype, int kind, const UpdateArgs& a, int width, cudaStream_t s) {
  const int64_t groups = a.dim / decode_channels_per_thread(kind, dtype);
  const int64_t rows = (int64_t)(CC1D_DECODE_THREADS / 32) * (kind == kDecodeRing ? CC1D_RING_ROWS : CC1D_DECODE_ROWS);
  const dim3 grid((unsigned)(((groups + 31) / 32) * ((a.batch + rows - 1) / rows)));
  switch (dtype) {
    case CC1D_FLOAT32: return launch_decode_t<float>(kind, a, width, grid, s);
    case CC1D_FLOAT16: return launch_decode_t<__half>(kind, a, width, grid, s);
    case CC1D_BFLOAT16: return launch_decode_t<__nv_bfloat16>(kind, a, width, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cc1d
