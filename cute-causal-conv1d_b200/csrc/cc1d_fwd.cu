// Forward kernels of the depthwise causal conv1d (sm_100a).
//
// Two layouts, both HBM-bound streaming stencils with fp32 accumulation and fused
// bias + SiLU:
//
//  * channel-last x (stride over dim == 1): a thread owns VEC consecutive channels
//    (one 16-byte packet) of one batch row and walks `chunk` sequence positions in
//    order, keeping the W-1 previous rows in registers, so every x row is read once
//    per chunk (plus a W-1 row halo at the chunk start).  A warp covers 32 packets
//    of one row: 512 contiguous bytes per load and per store.
//  * (batch, dim, seqlen)-contiguous x: a group of G lanes walks one channel row,
//    each lane holding VEC consecutive positions (one 16-byte packet); the W-1
//    element halo comes from the lane to the left with __shfl_up_sync and across
//    rounds from a carried register copy of the previous round's tail.
//
// Both kernels are persistent: the grid is sized to the resident CTA count and each
// CTA strides over tiles.  Compiled once per element type (CC1D_DT).
#include <climits>

#include "cc1d_common.cuh"
#include "cc1d_launch.h"

namespace cc1d {

// ------------------------------------------------------------- channel-last
template <typename T, int W, int VEC, bool SILU, bool SEQ, int U>
__global__ void __launch_bounds__(kThreads) fwd_channel_last_kernel(const ConvArgs a) {
  const int TX = 1 << a.tx_shift;
  const int tx = threadIdx.x & (TX - 1);
  const int ty = threadIdx.x >> a.tx_shift;
  const int TY = kThreads >> a.tx_shift;
  const int64_t L = a.seqlen;
  const int64_t ntiles = a.nbx * a.nby * a.batch;

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    int64_t t = tile;
    const int64_t bx = t % a.nbx;
    t /= a.nbx;
    const int64_t by = t % a.nby;
    const int64_t b = t / a.nby;
    const int64_t cv = bx * TX + tx;
    const int64_t l0 = (by * TY + ty) * a.chunk;
    if (cv >= a.nv || l0 >= L) continue;
    const int64_t l1 = min(l0 + a.chunk, L);
    const int64_t d0 = cv * VEC;

    float wv[W][VEC], bv[VEC];
    load_params<W, VEC>(a, d0, wv, bv);

    const T* xrow = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 * a.x.s1;
    T* orow = static_cast<T*>(a.out.data) + b * a.out.s0 + d0 * a.out.s1;
    const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;

    // x at positions l0-(W-1) .. l0-1 (initial states or zeros before 0).
    float xw[W - 1][VEC];
    int sw[W - 1];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
      const int64_t l = l0 - (W - 1) + k;
      if (l >= 0) {
        unpack<T, VEC>(ld_packet<T, VEC>(xrow + l * a.x.s2), xw[k]);
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v)
          xw[k][v] = a.init.data ? load_any(a.init.data, a.init.dtype,
                                            b * a.init.s0 + (d0 + v) * a.init.s1 + (W - 1 + l) * a.init.s2)
                                 : 0.f;
      }
      if constexpr (SEQ) sw[k] = l >= 0 ? srow[l * a.seq_idx.s1] : -1;
    }

    for (int64_t l = l0; l < l1; l += U) {
      Packet<T, VEC> raw[U];
      int sq[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (l + u < l1) raw[u] = ld_packet<T, VEC>(xrow + (l + u) * a.x.s2);
        if constexpr (SEQ) sq[u] = (l + u < l1) ? srow[(l + u) * a.seq_idx.s1] : -1;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (l + u < l1) {
          float xc[VEC];
          unpack<T, VEC>(raw[u], xc);
          float acc[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            float s = bv[v];
#pragma unroll
            for (int w = 0; w < W - 1; ++w) {
              float xin = xw[w][v];
              if constexpr (SEQ) xin = (sw[w] == sq[u]) ? xin : 0.f;
              s = fmaf(wv[w][v], xin, s);
            }
            s = fmaf(wv[W - 1][v], xc[v], s);
            if constexpr (SEQ) s = (sq[u] >= 0) ? s : 0.f;
            if constexpr (SILU) s = silu_fwd<T>(s);
            acc[v] = s;
          }
          st_packet<T, VEC>(orow + (l + u) * a.out.s2, pack<T, VEC>(acc));
#pragma unroll
          for (int k = 0; k < W - 2; ++k) {
#pragma unroll
            for (int v = 0; v < VEC; ++v) xw[k][v] = xw[k + 1][v];
            if constexpr (SEQ) sw[k] = sw[k + 1];
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) xw[W - 2][v] = xc[v];
          if constexpr (SEQ) sw[W - 2] = sq[u];
        }
      }
    }

    // The last chunk holds the final W-1 history entries in its window.
    if (a.final_states.data && l1 == L) {
#pragma unroll
      for (int k = 0; k < W - 1; ++k)
#pragma unroll
        for (int v = 0; v < VEC; ++v)
          store_any(a.final_states.data, a.final_states.dtype,
                    b * a.final_states.s0 + (d0 + v) * a.final_states.s1 + k * a.final_states.s2, xw[k][v]);
    }
  }
}

// ----------------------------------------------------- channel-last, streamed
// One wave of persistent warps (see WarpUnit): lane = one VEC-channel packet, warp =
// 32 consecutive packets of one batch row and one sequence segment [l0, l1).  The W-1 rows before l0 (or the
// initial states) are read once into the register window; rows l0 .. l1-1 then stream
// through a private ring of P shared-memory slots filled with cp.async, so P-1 rows per
// thread are in flight without occupying registers.  The row loop is unrolled by P
// (compile-time ring slots, window rotation by register renaming) and has no bounds
// checks; arithmetic runs on fp32 pairs (FFMA2).  With 16-bit SiLU the weights and
// bias are pre-scaled by 1/2 so the accumulator is h = p/2 and silu(p) = h*tanh(h) + h.
// Varlen decode states written by the streamed forward (EMIT).  The packed rows of
// sequence k are [cu[k], cu[k+1]); its state slot s holds x row cu[k+1] - S + s when
// that row is >= cu[k], else zero (the contract of varlen_states_kernel).  Each warp
// unit stores the slots of the rows it owns, from the packets it streams:
//  * the zero slots of a sequence shorter than S are written by the unit owning its
//    first row, when that unit makes the sequence current;
//  * an empty sequence is zero-filled by the unit owning the last row of the nearest
//    non-empty sequence before it, or, when there is none, by the unit holding row 0.
// Every field is the same for all lanes of the warp, so the tests are uniform; cu is
// read once per sequence (the next end is prefetched when a sequence becomes current).
// Writes stay inside states for any cu values: k < nseq and 0 <= slot < S always.
__device__ __forceinline__ int cu_row(const ConvArgs& a, int i) {
  const int64_t v = a.cu_is_64 ? __ldg(static_cast<const long long*>(a.cu) + i * a.cu_stride)
                               : static_cast<int64_t>(__ldg(static_cast<const int*>(a.cu) + i * a.cu_stride));
  return static_cast<int>(min(max(v, int64_t(-1)), a.seqlen + 1));
}

template <typename T, int VEC>
struct StateEmitter {
  T* chan;       // states + d0 (this lane's channel packet)
  int l0, l1;    // rows of this unit
  int k;         // current sequence
  int lo, hi;    // rows [lo, hi) of sequence k have a slot; lo == INT_MAX when done
  int next_end;  // cu[k + 2] (prefetched), or -2 past the last sequence
  int pre, pre0; // with nseq <= live lanes: cu[lane + 1] (cu[nseq] past the end) and cu[0]

  __device__ __forceinline__ T* slot(const ConvArgs& a, int kk, int s) const {
    return chan + kk * a.states.s0 + s * a.states.s2;
  }
  __device__ __forceinline__ void zero(const ConvArgs& a, int kk, int n) const {
    Packet<T, VEC> z;
#pragma unroll
    for (int v = 0; v < VEC; ++v) z.v[v] = from_f32<T>(0.f);
    for (int s = 0; s < n; ++s) st_packet<T, VEC>(slot(a, kk, s), z);
  }
  // Makes sequence kk (starting at row c0, ending at c1 when c1 >= -1 is given) or the
  // next non-empty one current; with `fill`, empty sequences passed over are zeroed.
  __device__ __forceinline__ void arm(const ConvArgs& a, int kk, int c0, int c1, bool fill) {
    for (; kk < a.nseq; ++kk) {
      if (c1 < -1) c1 = cu_row(a, kk + 1);
      if (c1 > c0) {
        k = kk;
        hi = c1;
        lo = max(c0, c1 - a.state_len);
        next_end = kk + 1 < a.nseq ? cu_row(a, kk + 2) : -2;
        if (c1 - c0 < a.state_len && c0 >= l0 && c0 < l1) zero(a, kk, a.state_len - (c1 - c0));
        return;
      }
      if (fill) zero(a, kk, a.state_len);
      c0 = c1;
      c1 = -2;
    }
    k = a.nseq;
    lo = hi = INT_MAX;
  }

  // Issued first in the kernel, before the row prefetch, so that the offsets have
  // arrived when start() needs them: with at most one sequence per live lane, lane j
  // loads cu[j + 1] and every lane cu[0].
  __device__ __forceinline__ void issue(const ConvArgs& a, int lane, int live) {
    if (a.nseq <= live) {
      pre = cu_row(a, min(lane, a.nseq - 1) + 1);
      pre0 = cu_row(a, 0);
    }
  }

  // The first sequence ending after row l0 becomes current.  Lanes 0 .. live-1 of the
  // warp take part (the others have left).  With nseq <= live the offsets loaded by
  // issue() give it with one ballot and two shuffles; otherwise, with 4 or more lanes,
  // each round probes `live` candidates at once and narrows the range by that factor,
  // else a binary search.
  __device__ __forceinline__ void start(const ConvArgs& a, int64_t d0, int first_row, int end_row, int lane,
                                        int live) {
    chan = static_cast<T*>(a.states.data) + d0 * a.states.s1;
    l0 = first_row;
    l1 = end_row;
    const unsigned mask = live >= 32 ? 0xffffffffu : (1u << live) - 1u;
    const bool row0 = l0 == 0;
    if (a.nseq <= live) {
      const unsigned hit = __ballot_sync(mask, pre > l0);  // lanes past nseq repeat cu[nseq]
      const int k0 = hit ? __ffs(hit) - 1 : a.nseq;
      const int c1 = __shfl_sync(mask, pre, min(k0, a.nseq - 1));
      const int c0 = __shfl_sync(mask, pre, max(k0 - 1, 0));
      if (row0)  // sequences ending at or before row 0 are empty and have no earlier owner
        for (int j = 0; j < k0; ++j) zero(a, j, a.state_len);
      arm(a, k0, k0 > 0 ? c0 : pre0, c1, row0);
      return;
    }
    int lo_k = 0, hi_k = a.nseq;  // the answer, first k with cu[k + 1] > l0 or nseq, is in [lo_k, hi_k]
    if (live >= 4) {
      while (lo_k < hi_k) {
        const int step = (hi_k - lo_k + live - 1) / live;
        const int c = min(lo_k + (lane + 1) * step, hi_k) - 1;  // last candidate of bucket `lane`
        const unsigned hit = __ballot_sync(mask, cu_row(a, c + 1) > l0);
        if (hit == 0) {
          lo_k = hi_k;
          break;
        }
        const int j = __ffs(hit) - 1;
        hi_k = min(lo_k + (j + 1) * step, hi_k) - 1;
        lo_k += j * step;
      }
    } else {
      while (lo_k < hi_k) {
        const int mid = (lo_k + hi_k) >> 1;
        if (cu_row(a, mid + 1) > l0) hi_k = mid; else lo_k = mid + 1;
      }
    }
    if (row0)
      for (int j = 0; j < lo_k; ++j) zero(a, j, a.state_len);
    arm(a, lo_k, lo_k < a.nseq ? cu_row(a, lo_k) : 0, -2, row0);
  }
  // Stores row l (streamed as `raw`) if it is a state row of the current sequence.
  __device__ __forceinline__ void store(const ConvArgs& a, int l, const Packet<T, VEC>& raw) const {
    if (l >= lo && l < hi) st_packet<T, VEC>(slot(a, k, l - (hi - a.state_len)), raw);
  }
  // Row-by-row form: stores row l and moves on after the current sequence's last row.
  __device__ __forceinline__ void row(const ConvArgs& a, int l, const Packet<T, VEC>& raw) {
    if (l < lo) return;
    store(a, l, raw);
    if (l == hi - 1) arm(a, k + 1, hi, next_end, true);
  }
  // Whether a block of rows ending at b1 (and starting at or after the rows already
  // passed) holds state rows of the current sequence only, so that it can store them
  // with store() and call after_block() once at its end.
  __device__ __forceinline__ bool one_sequence(const ConvArgs& a, int b1) const {
    return b1 < hi || next_end == -2 || next_end - a.state_len >= b1;
  }
  __device__ __forceinline__ void after_block(const ConvArgs& a, int b1) {
    if (b1 >= hi) arm(a, k + 1, hi, next_end, true);
  }
};

template <typename T, int W, int VEC, bool SILU, bool SEQ, int P, int NT, bool EMIT = false>
__global__ void __launch_bounds__(NT) fwd_stream_kernel(const ConvArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  using Pk = Packet<T, VEC>;
  constexpr int H = VEC / 2;
  constexpr bool HALF_ARG = SILU && !std::is_same<T, float>::value;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Pk* ring = reinterpret_cast<Pk*>(smem_raw) + threadIdx.x;  // slot s at ring[s * NT]
  const int lane = threadIdx.x & 31;
  // warps take units round robin over the CTAs, so that fewer units than resident warps
  // still spread over every SM (the host sizes the grid)
  const int64_t unit = (int64_t)(threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  if (unit >= a.units) return;
  const WarpUnit wu = warp_unit(a, unit);
  const int64_t pb = static_cast<unsigned>(wu.col) / static_cast<unsigned>(a.batch);  // packet block
  const int64_t b = wu.col - pb * a.batch;
  const int64_t cv = pb * 32 + lane;
  const int64_t L = a.seqlen;
  const int64_t l0 = part_start(wu.seg, wu.nseg, L);
  const int64_t l1 = part_start(wu.seg + 1, wu.nseg, L);
  if (cv >= a.nv || l0 >= l1) return;
  const int n = static_cast<int>(l1 - l0);
  const int64_t d0 = cv * VEC;
  const int64_t sx = a.x.s2, so = a.out.s2;
  const T* xsrc = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 + l0 * sx;
  [[maybe_unused]] StateEmitter<T, VEC> emit;
  [[maybe_unused]] const int live = static_cast<int>(min(a.nv - pb * 32, int64_t(32)));  // lanes left in the warp
  if constexpr (EMIT) emit.issue(a, lane, live);

  // prefetch rows l0 .. l0+P-2 before anything else (rows past the segment: zero fill)
#pragma unroll
  for (int j = 0; j < P - 1; ++j) {
    cp_async_packet<sizeof(Pk)>(ring + j * NT, xsrc, j < n);
    xsrc += sx;
    cp_async_commit();
  }

  // parameter and window loads are all issued before the first use of either
  float2 wv[W][H], bv[H];
  float2 xw[W - 1][H];
  {
    float wf[W][VEC], bf[VEC];
    load_params<W, VEC>(a, d0, wf, bf);
    load_window<T, W, VEC>(a, b, d0, l0, xw);
    const float sc = HALF_ARG ? 0.5f : 1.0f;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      bv[i] = make_float2(sc * bf[2 * i], sc * bf[2 * i + 1]);
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w][i] = make_float2(sc * wf[w][2 * i], sc * wf[w][2 * i + 1]);
    }
  }
  const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;
  int sw[W - 1];
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    const int64_t l = l0 - (W - 1) + k;
    sw[k] = (SEQ && l >= 0) ? srow[l * a.seq_idx.s1] : -1;
  }

  T* optr = static_cast<T*>(a.out.data) + b * a.out.s0 + d0 + l0 * so;
  // seq_idx: warps whose 32 lanes all hold channels (the others returned above) share
  // one coalesced load per 32 rows through SeqFeed's shuffles; a warp at the channel
  // edge, where some lanes have left, reads each row's value directly.
  const bool full_warp = (pb * 32 + 32) <= a.nv;  // the same for every lane of the warp
  SeqFeed seq;
  const int* sptr = SEQ ? srow + l0 * a.seq_idx.s1 : nullptr;
  if (SEQ && full_warp) seq.start(srow, a.seq_idx.s1, l0, L, lane);
  if constexpr (EMIT) emit.start(a, d0, static_cast<int>(l0), static_cast<int>(l1), lane, live);
  auto row = [&](const Pk& raw) {
    float2 xc[H];
    unpack2<T, VEC>(raw, xc);
    int scur = 0;
    if constexpr (SEQ) {
      if (full_warp) {
        scur = seq.next(lane);
      } else {
        scur = *sptr;
        sptr += a.seq_idx.s1;
      }
    }
    float2 acc[H];
#pragma unroll
    for (int i = 0; i < H; ++i) {
      float2 s = bv[i];
#pragma unroll
      for (int w = 0; w < W - 1; ++w) {
        float2 xin = xw[w][i];
        if constexpr (SEQ) xin = (sw[w] == scur) ? xin : make_float2(0.f, 0.f);
        s = ffma2(wv[w][i], xin, s);
      }
      s = ffma2(wv[W - 1][i], xc[i], s);
      if constexpr (SEQ) s = (scur >= 0) ? s : make_float2(0.f, 0.f);
      if constexpr (SILU) s = HALF_ARG ? silu_half_arg2(s) : silu_exact2(s);
      acc[i] = s;
    }
    st_packet<T, VEC>(optr, pack2<T, VEC>(acc));
    optr += so;
#pragma unroll
    for (int k = 0; k < W - 2; ++k) {
#pragma unroll
      for (int i = 0; i < H; ++i) xw[k][i] = xw[k + 1][i];
      sw[k] = sw[k + 1];
    }
#pragma unroll
    for (int i = 0; i < H; ++i) xw[W - 2][i] = xc[i];
    sw[W - 2] = scur;
  };
  // A row whose window rows all carry its own non-negative seq_idx: every mask is 1.
  [[maybe_unused]] auto row_same = [&](const Pk& raw) {
    float2 xc[H];
    unpack2<T, VEC>(raw, xc);
    float2 acc[H];
#pragma unroll
    for (int i = 0; i < H; ++i) {
      float2 s = bv[i];
#pragma unroll
      for (int w = 0; w < W - 1; ++w) s = ffma2(wv[w][i], xw[w][i], s);
      s = ffma2(wv[W - 1][i], xc[i], s);
      if constexpr (SILU) s = HALF_ARG ? silu_half_arg2(s) : silu_exact2(s);
      acc[i] = s;
    }
    st_packet<T, VEC>(optr, pack2<T, VEC>(acc));
    optr += so;
#pragma unroll
    for (int k = 0; k < W - 2; ++k)
#pragma unroll
      for (int i = 0; i < H; ++i) xw[k][i] = xw[k + 1][i];
#pragma unroll
    for (int i = 0; i < H; ++i) xw[W - 2][i] = xc[i];
  };
  int j0 = 0;
  if constexpr (EMIT) {
    // The plain loop below, written out again (the same text keeps the same code), up
    // to the next block holding state rows.  Such a block stores them from the ring;
    // the rare block that also reaches into the next sequence's state rows goes row
    // by row.
    for (;;) {
      const int64_t plain_end = min(static_cast<int64_t>(n), static_cast<int64_t>(emit.lo) - l0);
      for (; j0 + P <= plain_end; j0 += P) {
        if (full_warp) {  // one non-negative id over the block and its window: no masks
          const int v = sw[0];
          bool same = v >= 0;
#pragma unroll
          for (int w = 1; w < W - 1; ++w) same = same && sw[w] == v;
          if (same && seq.next_all(lane, P, v)) {  // `same` is the same in every lane
#pragma unroll
            for (int u = 0; u < P; ++u) {
              cp_async_packet<sizeof(Pk)>(ring + ((u + P - 1) % P) * NT, xsrc, j0 + u + P - 1 < n);
              xsrc += sx;
              cp_async_commit();
              cp_async_wait<P - 1>();
              row_same(ring[u * NT]);
            }
            seq.skip(lane, P);
            continue;
          }
        }
#pragma unroll
        for (int u = 0; u < P; ++u) {
          cp_async_packet<sizeof(Pk)>(ring + ((u + P - 1) % P) * NT, xsrc, j0 + u + P - 1 < n);
          xsrc += sx;
          cp_async_commit();
          cp_async_wait<P - 1>();
          row(ring[u * NT]);
        }
      }
      if (j0 + P > n) break;
      const int b1 = static_cast<int>(l0) + j0 + P;
      if (emit.one_sequence(a, b1)) {
#pragma unroll
        for (int u = 0; u < P; ++u) {
          cp_async_packet<sizeof(Pk)>(ring + ((u + P - 1) % P) * NT, xsrc, j0 + u + P - 1 < n);
          xsrc += sx;
          cp_async_commit();
          cp_async_wait<P - 1>();
          emit.store(a, static_cast<int>(l0) + j0 + u, ring[u * NT]);
          row(ring[u * NT]);
        }
        emit.after_block(a, b1);
        j0 += P;
      } else {
        for (const int j1 = j0 + P; j0 < j1; ++j0) {
          cp_async_packet<sizeof(Pk)>(ring + ((j0 + P - 1) % P) * NT, xsrc, j0 + P - 1 < n);
          xsrc += sx;
          cp_async_commit();
          cp_async_wait<P - 1>();
          emit.row(a, static_cast<int>(l0) + j0, ring[(j0 % P) * NT]);
          row(ring[(j0 % P) * NT]);
        }
      }
    }
    for (int j = j0; j < n; ++j) {  // remainder
      cp_async_packet<sizeof(Pk)>(ring + ((j + P - 1) % P) * NT, xsrc, j + P - 1 < n);
      xsrc += sx;
      cp_async_commit();
      cp_async_wait<P - 1>();
      emit.row(a, static_cast<int>(l0) + j, ring[(j % P) * NT]);
      row(ring[(j % P) * NT]);
    }
  } else {
    // full blocks of P rows: compile-time ring slots, predicated prefetch, no branches.
    // With seq_idx, a full warp runs a block whose P rows and W-1 window rows all carry
    // one non-negative id without the masks (the same result).
    for (; j0 + P <= n; j0 += P) {
      if constexpr (SEQ) {
        if (full_warp) {
          const int v = sw[0];
          bool same = v >= 0;
#pragma unroll
          for (int w = 1; w < W - 1; ++w) same = same && sw[w] == v;
          if (same && seq.next_all(lane, P, v)) {  // `same` is the same in every lane
#pragma unroll
            for (int u = 0; u < P; ++u) {
              cp_async_packet<sizeof(Pk)>(ring + ((u + P - 1) % P) * NT, xsrc, j0 + u + P - 1 < n);
              xsrc += sx;
              cp_async_commit();
              cp_async_wait<P - 1>();
              row_same(ring[u * NT]);
            }
            seq.skip(lane, P);
            continue;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < P; ++u) {
        cp_async_packet<sizeof(Pk)>(ring + ((u + P - 1) % P) * NT, xsrc, j0 + u + P - 1 < n);
        xsrc += sx;
        cp_async_commit();
        cp_async_wait<P - 1>();
        row(ring[u * NT]);
      }
    }
    for (int j = j0; j < n; ++j) {  // remainder
      cp_async_packet<sizeof(Pk)>(ring + ((j + P - 1) % P) * NT, xsrc, j + P - 1 < n);
      xsrc += sx;
      cp_async_commit();
      cp_async_wait<P - 1>();
      row(ring[(j % P) * NT]);
    }
  }
  cp_async_wait<0>();

  if (a.final_states.data && l0 + n == L) {
#pragma unroll
    for (int k = 0; k < W - 1; ++k)
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const int64_t o = b * a.final_states.s0 + (d0 + 2 * i) * a.final_states.s1 + k * a.final_states.s2;
        store_any(a.final_states.data, a.final_states.dtype, o, xw[k][i].x);
        store_any(a.final_states.data, a.final_states.dtype, o + a.final_states.s1, xw[k][i].y);
      }
  }
}

// ------------------------------------------------------------------- rows
// Value of element `idx` (0 <= idx < W-1, run-time) of a W-1 register array.
template <int N, typename V>
__device__ __forceinline__ V pick(const V (&arr)[N], int idx) {
  V r = arr[0];
#pragma unroll
  for (int q = 1; q < N; ++q) r = (idx == q) ? arr[q] : r;
  return r;
}

template <typename T, int W, int VEC, bool SILU, bool SEQ>
__global__ void __launch_bounds__(kThreads) fwd_row_kernel(const ConvArgs a) {
  constexpr unsigned FULL = 0xffffffffu;
  const int G = 1 << a.g_shift;
  const int gl = threadIdx.x & (G - 1);
  const int group = threadIdx.x >> a.g_shift;
  const int DPB = kThreads >> a.g_shift;
  const int64_t L = a.seqlen;
  const int64_t span = (int64_t)G * VEC;
  const int64_t ntiles = a.nbx * a.nck * a.batch;

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    int64_t t = tile;
    const int64_t dtile = t % a.nbx;
    t /= a.nbx;
    const int64_t c = t % a.nck;
    const int64_t b = t / a.nck;
    const int64_t d = dtile * DPB + group;
    const bool row_ok = d < a.dim;
    const int64_t dd = row_ok ? d : 0;
    const int64_t cs = c * a.chunk;
    const int64_t ce = min(cs + a.chunk, L);

    const T* xrow = static_cast<const T*>(a.x.data) + b * a.x.s0 + dd * a.x.s1;
    T* orow = static_cast<T*>(a.out.data) + b * a.out.s0 + dd * a.out.s1;
    const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;

    float wv[W], bias;
    {
      float wt[W][1], bt[1];
      load_params<W, 1>(a, dd, wt, bt);
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w] = wt[w][0];
      bias = bt[0];
    }

    // carry[j] = x at cs-(W-1)+j ; scarry likewise for seq_idx
    float carry[W - 1];
    int scarry[W - 1];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const int64_t pos = cs - (W - 1) + j;
      float v = 0.f;
      if (row_ok) {
        if (pos >= 0) v = to_f32(xrow[pos * a.x.s2]);
        else if (a.init.data)
          v = load_any(a.init.data, a.init.dtype, b * a.init.s0 + dd * a.init.s1 + (W - 1 + pos) * a.init.s2);
      }
      carry[j] = v;
      if constexpr (SEQ) scarry[j] = (row_ok && pos >= 0) ? srow[pos * a.seq_idx.s1] : -1;
    }

    for (int r = 0; r < a.rounds; ++r) {
      const int64_t e0 = cs + r * span + gl * VEC;
      float xv[VEC];
      int sv[VEC];
      if (row_ok && e0 + VEC <= ce) {
        unpack<T, VEC>(ld_packet<T, VEC>(xrow + e0), xv);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) xv[i] = (row_ok && e0 + i < ce) ? to_f32(xrow[e0 + i]) : 0.f;
      }
      if constexpr (SEQ) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) sv[i] = (row_ok && e0 + i < ce) ? srow[(e0 + i) * a.seq_idx.s1] : -1;
      }
      // xs[q] = x at e0 - (W-1) + q
      float xs[VEC + W - 1];
      int ss[VEC + W - 1];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        xs[W - 1 + i] = xv[i];
        if constexpr (SEQ) ss[W - 1 + i] = sv[i];
      }
#pragma unroll
      for (int k = 1; k < W; ++k) {
        const int delta = (k + VEC - 1) / VEC;
        const int slot = delta * VEC - k;
        float hv = __shfl_up_sync(FULL, xv[slot], delta, G);
        int hs = 0;
        if constexpr (SEQ) hs = __shfl_up_sync(FULL, sv[slot], delta, G);
        if (gl < delta) {
          const int idx = W - 1 - k + gl * VEC;
          hv = pick<W - 1>(carry, idx);
          if constexpr (SEQ) hs = pick<W - 1>(scarry, idx);
        }
        xs[W - 1 - k] = hv;
        if constexpr (SEQ) ss[W - 1 - k] = hs;
      }
      float acc[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        float s = bias;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          float xin = xs[i + w];
          if constexpr (SEQ) xin = (ss[i + w] == ss[W - 1 + i]) ? xin : 0.f;
          s = fmaf(wv[w], xin, s);
        }
        if constexpr (SEQ) s = (ss[W - 1 + i] >= 0) ? s : 0.f;
        if constexpr (SILU) s = silu_fwd<T>(s);
        acc[i] = s;
      }
      if (row_ok && e0 + VEC <= ce) {
        st_packet<T, VEC>(orow + e0, pack<T, VEC>(acc));
      } else if (row_ok) {
#pragma unroll
        for (int i = 0; i < VEC; ++i)
          if (e0 + i < ce) orow[e0 + i] = from_f32<T>(acc[i]);
      }
      // carry = last W-1 elements of this round (the round spans >= W-1 elements)
#pragma unroll
      for (int j = 0; j < W - 1; ++j) {
        const int m = W - 1 - j;
        const int delta = (m + VEC - 1) / VEC;
        const int slot = delta * VEC - m;
        carry[j] = __shfl_sync(FULL, xv[slot], G - delta, G);
        if constexpr (SEQ) scarry[j] = __shfl_sync(FULL, sv[slot], G - delta, G);
      }
    }

    // final states: last W-1 entries of [initial | x], reread from memory.
    if (a.final_states.data && row_ok && c == a.nck - 1 && gl < W - 1) {
      const int64_t pos = L - (W - 1) + gl;
      float v = 0.f;
      if (pos >= 0) v = to_f32(xrow[pos * a.x.s2]);
      else if (a.init.data)
        v = load_any(a.init.data, a.init.dtype, b * a.init.s0 + d * a.init.s1 + (W - 1 + pos) * a.init.s2);
      store_any(a.final_states.data, a.final_states.dtype,
                b * a.final_states.s0 + d * a.final_states.s1 + gl * a.final_states.s2, v);
    }
  }
}

// ----------------------------------------------------------------- dispatch
template <typename T, int W, int VEC>
static cudaError_t launch_fwd_w(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  const bool silu = ls.silu, seq = ls.seq;
  if (ls.layout == kLayoutStream) {
    if constexpr (VEC * sizeof(T) == kFwdPacketBytes) {
#define CC1D_GO_P(SI, SQ, EM, P, NT)                                                                \
  do {                                                                                              \
    const auto kern = fwd_stream_kernel<T, W, VEC, SI, SQ, P, NT, EM>;                              \
    const cudaError_t ea = allow_dynamic_smem(reinterpret_cast<const void*>(kern), ls.smem);       \
    if (ea != cudaSuccess) return ea;                                                               \
    return launch_dependent(kern, ls.grid, dim3(NT), ls.smem, s, a);                                \
  } while (0)
#define CC1D_GO(SI, SQ, EM)                                                                         \
  CC1D_GO_P(SI, SQ, EM, (EM ? kStreamDepthEmit : kStreamDepthFwd), kFwdStreamThreads)
#define CC1D_GO_SMALL(SI, SQ) CC1D_GO_P(SI, SQ, false, kStreamDepthFwdSmall, kFwdStreamThreadsSmall)
      // The state-emitting variant keeps 8-slot rings: with 16-row blocks it ran 362 us
      // instead of 252 us on 1024 packed sequences of 64 rows (config 4's shape).
      if (ls.emit) {  // packed sequences: seq_idx is present
        if (silu) CC1D_GO(true, true, true); else CC1D_GO(false, true, true);
      }
      if (ls.small) {
        if (silu) { if (seq) CC1D_GO_SMALL(true, true); else CC1D_GO_SMALL(true, false); }
        else { if (seq) CC1D_GO_SMALL(false, true); else CC1D_GO_SMALL(false, false); }
      }
      if (silu) { if (seq) CC1D_GO(true, true, false); else CC1D_GO(true, false, false); }
      else { if (seq) CC1D_GO(false, true, false); else CC1D_GO(false, false, false); }
#undef CC1D_GO_SMALL
#undef CC1D_GO
#undef CC1D_GO_P
    }
  } else if (ls.layout == kLayoutChannelLast) {
    constexpr int U = 4;
#define CC1D_GO(SI, SQ) fwd_channel_last_kernel<T, W, VEC, SI, SQ, U><<<ls.grid, kThreads, 0, s>>>(a)
    if (silu) { if (seq) CC1D_GO(true, true); else CC1D_GO(true, false); }
    else { if (seq) CC1D_GO(false, true); else CC1D_GO(false, false); }
#undef CC1D_GO
  } else {
#define CC1D_GO(SI, SQ) fwd_row_kernel<T, W, VEC, SI, SQ><<<ls.grid, kThreads, 0, s>>>(a)
    if (silu) { if (seq) CC1D_GO(true, true); else CC1D_GO(true, false); }
    else { if (seq) CC1D_GO(false, true); else CC1D_GO(false, false); }
#undef CC1D_GO
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_fwd_t(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  constexpr int PV = 16 / sizeof(T);
  constexpr int SV = kFwdPacketBytes / sizeof(T);  // the streamed kernel's packets
  if (ls.layout == kLayoutStream) {
    switch (ls.width) {
      case 2: return launch_fwd_w<T, 2, SV>(a, ls, s);
      case 3: return launch_fwd_w<T, 3, SV>(a, ls, s);
      case 4: return launch_fwd_w<T, 4, SV>(a, ls, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (ls.width * 2 + (ls.packet ? 1 : 0)) {
    case 4: return launch_fwd_w<T, 2, 1>(a, ls, s);
    case 5: return launch_fwd_w<T, 2, PV>(a, ls, s);
    case 6: return launch_fwd_w<T, 3, 1>(a, ls, s);
    case 7: return launch_fwd_w<T, 3, PV>(a, ls, s);
    case 8: return launch_fwd_w<T, 4, 1>(a, ls, s);
    case 9: return launch_fwd_w<T, 4, PV>(a, ls, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static const void* fwd_kernel_ptr_t(const LaunchShape& ls) {
  // Any instantiation of the same family has the same resource footprint class; the
  // host uses this only for occupancy queries.
  constexpr int PV = 16 / sizeof(T);
  if (ls.layout == kLayoutStream && ls.small)
    return reinterpret_cast<const void*>(
        fwd_stream_kernel<T, 4, kFwdPacketBytes / sizeof(T), true, false, kStreamDepthFwdSmall, kFwdStreamThreadsSmall>);
  if (ls.layout == kLayoutStream)
    return reinterpret_cast<const void*>(
        fwd_stream_kernel<T, 4, kFwdPacketBytes / sizeof(T), true, false, kStreamDepthFwd, kFwdStreamThreads>);
  if (ls.layout == kLayoutChannelLast) {
    if (ls.packet) return reinterpret_cast<const void*>(fwd_channel_last_kernel<T, 4, PV, true, false, 4>);
    return reinterpret_cast<const void*>(fwd_channel_last_kernel<T, 4, 1, true, false, 4>);
  }
  if (ls.packet) return reinterpret_cast<const void*>(fwd_row_kernel<T, 4, PV, true, false>);
  return reinterpret_cast<const void*>(fwd_row_kernel<T, 4, 1, true, false>);
}

cudaError_t CC1D_DT_NAME(fwd)(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  return launch_fwd_t<CC1D_DT_TYPE>(a, ls, s);
}

const void* CC1D_DT_NAME(fwd_kernel_ptr)(const LaunchShape& ls) {
  return fwd_kernel_ptr_t<CC1D_DT_TYPE>(ls);
}

}  // namespace cc1d
