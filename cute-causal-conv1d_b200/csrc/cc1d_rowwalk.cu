// Row-walk forward and backward kernels for (batch, dim, seqlen)-contiguous tensors
// (sm_100a).  Compiled once per element type (CC1D_DT).
//
// A row is one (b, d) pair; rows are numbered channel-major (row = d * batch + b) so that
// the rows of one channel are consecutive.  A step is 32 lanes x VEC consecutive
// positions of one row (VEC elements = one aligned 16-byte packet per lane): a warp
// reads 512 contiguous bytes per step and per tensor.  The steps of all rows, row after
// row, form one sequence of a.units steps; warp w of the a.ncol warps of the grid (one
// wave) walks the contiguous range [part_start(w), part_start(w + 1)) of it.  Ranges
// start and end inside rows and run across row boundaries, so every warp gets the same
// number of steps (+-1), and the warp's private cp.async ring (P slots per lane and
// tensor, zero-filled past the range and past the row end) keeps streaming across row
// boundaries without refilling.
//
// The W-1 positions left of a lane's packet come from the previous lane
// (__shfl_up_sync); lane 0 takes them from a register carry (lane 31 of the previous
// step, the initial states at position 0, or a direct load where a range starts inside
// a row).  The backward emits dx one step late: dx needs g at the W-1 positions right of
// a packet, which come from the next lane (__shfl_down_sync) or, for lane 31, from
// lane 0 of the next step.  A range that ends inside a row walks one more step (loads,
// no accumulation) to obtain those g values.
//
// dweight/dbias: each warp keeps fp32 pair sums per channel; when the channel changes and
// at the end of its range it reduces them over its lanes (fixed butterfly) and lane 0
// writes W+1 floats to slot (d + w) - distinct for every (channel, warp) piece because
// both the channel ranges and the warp ranges are contiguous and ordered.
// reduce_rowwalk_partials then adds the pieces of each channel in warp order: the sums
// do not depend on scheduling.
#include "cc1d_common.cuh"
#include "cc1d_launch.h"

namespace cc1d {

// Position of a warp in the step sequence.
struct RowCursor {
  int step, b, d;  // step within the row, and the row's batch index and channel (the
                   // planner keeps rows x steps below 2^31)
};
__device__ __forceinline__ RowCursor cursor_at(const ConvArgs& a, int64_t q) {
  RowCursor c;
  const int64_t row = q / a.nck;
  c.step = static_cast<int>(q - row * a.nck);
  c.d = static_cast<int>(row / a.batch);
  c.b = static_cast<int>(row - (int64_t)c.d * a.batch);
  return c;
}
__device__ __forceinline__ void cursor_next(RowCursor& c, const ConvArgs& a) {
  if (++c.step == a.nck) {
    c.step = 0;
    if (++c.b == a.batch) {
      c.b = 0;
      ++c.d;
    }
  }
}
template <typename T>
__device__ __forceinline__ T* row_of(const TensorArg& t, const RowCursor& c) {
  return static_cast<T*>(t.data) + (int64_t)c.b * t.s0 + (int64_t)c.d * t.s1;
}

// The W-1 values of x left of position p0 of the cursor's row: initial states (or zero)
// left of position 0.
template <typename T, int W>
__device__ __forceinline__ void row_halo(const ConvArgs& a, const RowCursor& c, int64_t p0, float (&carry)[W - 1]) {
  const T* xrow = row_of<const T>(a.x, c);
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {
    const int64_t pos = p0 - (W - 1) + j;
    float v = 0.f;
    if (pos >= 0) v = to_f32(xrow[pos]);
    else if (a.init.data) v = load_any(a.init.data, a.init.dtype, (int64_t)c.b * a.init.s0 + (int64_t)c.d * a.init.s1 + (W - 1 + pos) * a.init.s2);
    carry[j] = v;
  }
}

// The row after c's row, at step 0.
__device__ __forceinline__ RowCursor row_after(const ConvArgs& a, RowCursor c) {
  c.step = 0;
  if (++c.b == a.batch) {
    c.b = 0;
    ++c.d;
  }
  return c;
}

// Initial states of row c (W-1 values, zero without initial_states or past the last row).
template <int W>
__device__ __forceinline__ void row_init(const ConvArgs& a, const RowCursor& c, float (&v)[W - 1]) {
  const bool ok = a.init.data && c.d < a.dim;
#pragma unroll
  for (int j = 0; j < W - 1; ++j)
    v[j] = ok ? load_any(a.init.data, a.init.dtype, (int64_t)c.b * a.init.s0 + (int64_t)c.d * a.init.s1 + j * a.init.s2) : 0.f;
}

// Weights and bias of channel d (scaled by sc; zero past the last channel).
template <int W>
__device__ __forceinline__ void channel_params(const ConvArgs& a, int64_t d, float sc, float (&wv)[W], float& bv) {
  if (d >= a.dim) {
#pragma unroll
    for (int w = 0; w < W; ++w) wv[w] = 0.f;
    bv = 0.f;
    return;
  }
  float wt[W][1], bt[1];
  load_params<W, 1>(a, d, wt, bt);
#pragma unroll
  for (int w = 0; w < W; ++w) wv[w] = sc * wt[w][0];
  bv = sc * bt[0];
}

// v[idx] for a run-time idx of a small register array (a select chain, no local memory).
template <int N>
__device__ __forceinline__ float select_of(const float (&v)[N], int64_t idx) {
  float r = v[0];
#pragma unroll
  for (int k = 1; k < N; ++k) r = idx == k ? v[k] : r;
  return r;
}

// x window of one lane: xs[k] = x at p0 - (W-1) + k (k < VEC + W - 1); carry (used by
// lane 0) becomes the last W-1 values of lane 31.  ROTATE: one rotation by a lane serves
// both (lane l > 0 receives the tail of lane l-1, lane 0 the tail of lane 31 for the
// next step); otherwise a shift up plus a broadcast of lane 31 (the forward keeps this
// form: the rotation saved it nothing).
template <int W, int VEC, bool ROTATE>
__device__ __forceinline__ void lane_window(const float (&xe)[VEC], float (&carry)[W - 1], int lane,
                                            float (&xs)[VEC + W - 1]) {
  constexpr unsigned FULL = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < VEC; ++i) xs[W - 1 + i] = xe[i];
  if constexpr (ROTATE) {
    const int left = (lane + 31) & 31;
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const float v = __shfl_sync(FULL, xe[VEC - (W - 1) + j], left);
      xs[j] = lane == 0 ? carry[j] : v;
      carry[j] = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const float v = __shfl_up_sync(FULL, xe[VEC - (W - 1) + j], 1);
      xs[j] = lane == 0 ? carry[j] : v;
    }
#pragma unroll
    for (int j = 0; j < W - 1; ++j) carry[j] = __shfl_sync(FULL, xe[VEC - (W - 1) + j], 31);
  }
}

// Producer side of the walk: streams this lane's packet of consecutive steps (running
// across rows) into a ring of P slots, zero-filling past the range and past the row end.
template <typename T, int VEC, int P, int NT, int NTENS>
struct WalkFeed {
  static constexpr int S = 32 * VEC;
  const TensorArg* tens[NTENS];
  Packet<T, VEC>* ring[NTENS];  // slot 0 of this thread's ring in each tensor
  const T* src[NTENS];          // this lane's packet of the next step
  int64_t pos;                  // its position in the row
  int step, b, d, slot, left;

  __device__ __forceinline__ void start(const ConvArgs& a, const RowCursor& c, int lane, int count) {
    step = c.step;
    b = c.b;
    d = c.d;
    slot = 0;
    left = count;
    pos = (int64_t)step * S + lane * VEC;
#pragma unroll
    for (int t = 0; t < NTENS; ++t) src[t] = static_cast<const T*>(tens[t]->data) + (int64_t)b * tens[t]->s0 + (int64_t)d * tens[t]->s1 + pos;
  }
  __device__ __forceinline__ void issue(const ConvArgs& a, int lane) {
    const bool ok = left > 0 && pos < a.seqlen;
#pragma unroll
    for (int t = 0; t < NTENS; ++t) cp_async_packet<sizeof(Packet<T, VEC>)>(ring[t] + slot * NT, src[t], ok);
    cp_async_commit();
    --left;
    slot = slot + 1 == P ? 0 : slot + 1;
    pos += S;
#pragma unroll
    for (int t = 0; t < NTENS; ++t) src[t] += S;
    if (++step == a.nck) {  // next row
      step = 0;
      if (++b == a.batch) {
        b = 0;
        ++d;
      }
      pos = lane * VEC;
#pragma unroll
      for (int t = 0; t < NTENS; ++t) src[t] = static_cast<const T*>(tens[t]->data) + (int64_t)b * tens[t]->s0 + (int64_t)d * tens[t]->s1 + pos;
    }
  }
};

// ------------------------------------------------------------------- forward
// STATES: initial_states and/or final_states are given (compiled out otherwise).
template <typename T, int W, bool SILU, bool STATES, int P, int NT>
__global__ void __launch_bounds__(NT) fwd_rowwalk_kernel(const ConvArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  constexpr int VEC = 16 / sizeof(T);
  constexpr int H2 = VEC / 2;
  constexpr int S = 32 * VEC;
  constexpr bool HALF_ARG = SILU && !std::is_same<T, float>::value;
  using Pk = Packet<T, VEC>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (warp >= a.ncol) return;
  const int64_t q0 = part_start(warp, a.ncol, a.units), q1 = part_start(warp + 1, a.ncol, a.units);
  if (q0 >= q1) return;
  const int n = static_cast<int>(q1 - q0);
  const int64_t L = a.seqlen;

  RowCursor cc = cursor_at(a, q0);
  WalkFeed<T, VEC, P, NT, 1> feed;
  feed.tens[0] = &a.x;
  feed.ring[0] = reinterpret_cast<Pk*>(smem_raw) + threadIdx.x;
  feed.start(a, cc, lane, n);
#pragma unroll
  for (int j = 0; j < P - 1; ++j) feed.issue(a, lane);

  // Row-boundary values are loaded one row (initial states) or one channel (weights)
  // ahead, so that no load latency sits on the walk.
  const float sc = HALF_ARG ? 0.5f : 1.0f;
  float wv[W], bv, wn[W], bn;
  int cur_d = cc.d;
  channel_params<W>(a, cc.d, sc, wv, bv);
  channel_params<W>(a, cc.d + 1, sc, wn, bn);
  float carry[W - 1], ninit[W - 1];
  row_halo<T, W>(a, cc, (int64_t)cc.step * S, carry);
  if constexpr (STATES) row_init<W>(a, row_after(a, cc), ninit);

  const Pk* ring = feed.ring[0];
  int slot = 0;
  int left = n;
  bool started = false;  // the first row's values come from the prologue
  while (left > 0) {
    if (cc.step == 0 && started) {  // a new row: take the values loaded ahead
#pragma unroll
      for (int j = 0; j < W - 1; ++j) carry[j] = STATES ? ninit[j] : 0.f;
      if constexpr (STATES) row_init<W>(a, row_after(a, cc), ninit);
      if (cc.d != cur_d) {
#pragma unroll
        for (int w = 0; w < W; ++w) wv[w] = wn[w];
        bv = bn;
        cur_d = cc.d;
        channel_params<W>(a, cc.d + 1, sc, wn, bn);
      }
    }
    started = true;
    const int seg = min(static_cast<int>(a.nck) - cc.step, left);
    const bool row_ends = cc.step + seg == a.nck;
    int64_t pos = (int64_t)cc.step * S + lane * VEC;
    T* po = row_of<T>(a.out, cc) + pos;
#pragma unroll 2
    for (int k = 0; k < seg; ++k) {
      feed.issue(a, lane);
      cp_async_wait<P - 1>();
      float xe[VEC], xs[VEC + W - 1];
      unpack<T, VEC>(ring[slot * NT], xe);
      slot = slot + 1 == P ? 0 : slot + 1;
      lane_window<W, VEC, false>(xe, carry, lane, xs);
      // fp32 pairs hold elements (m, m + VEC/2): a window shifted by w is again a pair
      // of the same layout, so no register has to be moved to form FFMA2 operands
      float o[VEC];
#pragma unroll
      for (int m = 0; m < H2; ++m) {
        float2 s = make_float2(bv, bv);
#pragma unroll
        for (int w = 0; w < W; ++w) s = ffma2(make_float2(wv[w], wv[w]), make_float2(xs[m + w], xs[m + H2 + w]), s);
        if constexpr (HALF_ARG) s = silu_half_arg2(s);
        else if constexpr (SILU) s = silu_exact2(s);
        o[m] = s.x;
        o[m + H2] = s.y;
      }
      if (pos < L) st_packet<T, VEC>(po, pack<T, VEC>(o));
      // final states: the last W-1 entries of x (seqlen is a whole number of packets >=
      // W-1, so they sit at the end of one lane's packet of the row's last step)
      if (STATES && a.final_states.data && row_ends && k == seg - 1) {
        const int src = static_cast<int>(((L - 1) % S) / VEC);
        float f[W - 1];
#pragma unroll
        for (int j = 0; j < W - 1; ++j) f[j] = __shfl_sync(0xffffffffu, xe[VEC - (W - 1) + j], src);
        if (lane < W - 1)
          store_any(a.final_states.data, a.final_states.dtype,
                    (int64_t)cc.b * a.final_states.s0 + (int64_t)cc.d * a.final_states.s1 + lane * a.final_states.s2,
                    select_of<W - 1>(f, lane));
      }
      pos += S;
      po += S;
    }
    left -= seg;
    cc.step += seg;
    if (cc.step == a.nck) {
      cc.step = 0;
      if (++cc.b == a.batch) {
        cc.b = 0;
        ++cc.d;
      }
    }
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ backward
// STATES: initial_states, dinitial_states and/or dfinal_states are given.
template <typename T, int W, bool SILU, bool STATES, int P, int NT>
__global__ void __launch_bounds__(NT) bwd_rowwalk_kernel(const ConvArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  constexpr int VEC = 16 / sizeof(T);
  constexpr int H2 = VEC / 2;  // fp32 pairs hold elements (m, m + H2), as in the forward
  constexpr int S = 32 * VEC;
  constexpr unsigned FULL = 0xffffffffu;
  // 16-bit tensors with SiLU: weights and bias are halved, the running sum is h = p/2
  // and g holds 2 * dout * silu'(p); dx = sum (w/2) g is exact and the dweight/dbias sums
  // carry a factor 2 removed when they are written.
  constexpr bool HALF = SILU && sizeof(T) == 2;
  using Pk = Packet<T, VEC>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (warp >= a.ncol) return;
  const int64_t q0 = part_start(warp, a.ncol, a.units), q1 = part_start(warp + 1, a.ncol, a.units);
  if (q0 >= q1) return;
  const int n = static_cast<int>(q1 - q0);  // steps that accumulate
  const bool halo_step = (q1 % a.nck) != 0; // the range ends inside a row: one more step
  const int64_t L = a.seqlen;

  RowCursor cc = cursor_at(a, q0);
  WalkFeed<T, VEC, P, NT, 2> feed;
  feed.tens[0] = &a.x;
  feed.tens[1] = &a.dout;
  feed.ring[0] = reinterpret_cast<Pk*>(smem_raw) + threadIdx.x;
  feed.ring[1] = reinterpret_cast<Pk*>(smem_raw) + P * NT + threadIdx.x;
  feed.start(a, cc, lane, n + (halo_step ? 1 : 0));
#pragma unroll
  for (int j = 0; j < P - 1; ++j) feed.issue(a, lane);

  // Row-boundary values are loaded one row (initial states, dfinal_states) or one
  // channel (weights) ahead, so that no load latency sits on the walk.
  constexpr float sc = HALF ? 0.5f : 1.0f;
  float wv[W], bv, wn[W], bn;
  int cur_d = cc.d;
  channel_params<W>(a, cc.d, sc, wv, bv);
  channel_params<W>(a, cc.d + 1, sc, wn, bn);
  float2 dw[W], db = make_float2(0.f, 0.f);
#pragma unroll
  for (int w = 0; w < W; ++w) dw[w] = make_float2(0.f, 0.f);
  float carry[W - 1], ninit[W - 1], dfin[W - 1];
  row_halo<T, W>(a, cc, (int64_t)cc.step * S, carry);
  if constexpr (STATES) row_init<W>(a, row_after(a, cc), ninit);
  auto row_dfinal = [&](const RowCursor& c) {
#pragma unroll
    for (int j = 0; j < W - 1; ++j)
      dfin[j] = a.dfinal.data ? load_any(a.dfinal.data, a.dfinal.dtype, (int64_t)c.b * a.dfinal.s0 + (int64_t)c.d * a.dfinal.s1 + j * a.dfinal.s2) : 0.f;
  };
  if constexpr (STATES) row_dfinal(cc);

  // this warp's (channel, range) piece of dweight/dbias
  auto flush = [&](int64_t d) {
    float v[W + 1];
#pragma unroll
    for (int w = 0; w < W; ++w) v[w] = sc * (dw[w].x + dw[w].y);
    v[W] = sc * (db.x + db.y);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int k = 0; k <= W; ++k) v[k] += __shfl_xor_sync(FULL, v[k], off);
    }
    if (lane == 0) {
      float* slot = a.partials + (d + warp) * (W + 1);
#pragma unroll
      for (int k = 0; k <= W; ++k) slot[k] = v[k];
    }
#pragma unroll
    for (int w = 0; w < W; ++w) dw[w] = make_float2(0.f, 0.f);
    db = make_float2(0.f, 0.f);
  };

  // dx of one step (g values gs, lane position pos, output pdx) given the first W-1 g
  // values of the step to its right (nxt, read from lane 0); on the row's last step
  // (last) it adds dfinal_states.  The right halo comes from one rotation by a lane:
  // rot_nxt (nxt of lane l+1) serves lane 31 now, and lanes 0..30 at the next step,
  // whose own g is this step's nxt; rot_gs holds that rotation of gs from the step before.
  const int right = (lane + 1) & 31;
  float rot_gs[W - 1];
  auto emit = [&](T* pdx, int64_t pos, const float (&gs)[VEC], const float (&nxt)[VEC], bool last) {
    float G[VEC + W - 1];
#pragma unroll
    for (int i = 0; i < VEC; ++i) G[i] = gs[i];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const float h = __shfl_sync(FULL, nxt[j], right);
      G[VEC + j] = lane == 31 ? h : rot_gs[j];
      rot_gs[j] = h;
    }
    float dxe[VEC];
#pragma unroll
    for (int m = 0; m < H2; ++m) {
      float2 s = make_float2(0.f, 0.f);
#pragma unroll
      for (int w = 0; w < W; ++w)
        s = ffma2(make_float2(wv[w], wv[w]), make_float2(G[m + W - 1 - w], G[m + H2 + W - 1 - w]), s);
      dxe[m] = s.x;
      dxe[m + H2] = s.y;
    }
    if (STATES && last && a.dfinal.data) {  // dfin: this row's dfinal_states
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int64_t jj = pos + e - (L - (W - 1));  // index into dfinal_states
        if (jj >= 0 && jj < W - 1) dxe[e] += select_of<W - 1>(dfin, jj);
      }
    }
    if (pos < L) st_packet<T, VEC>(pdx, pack<T, VEC>(dxe));
  };

  // g of the next ring slot (and its x window)
  const Pk* xring = feed.ring[0];
  const Pk* gring = feed.ring[1];
  int slot = 0;
  auto next_g = [&](float (&xs)[VEC + W - 1], float (&g)[VEC]) {
    feed.issue(a, lane);
    cp_async_wait<P - 1>();
    float xe[VEC], de[VEC];
    unpack<T, VEC>(xring[slot * NT], xe);
    unpack<T, VEC>(gring[slot * NT], de);
    slot = slot + 1 == P ? 0 : slot + 1;
    lane_window<W, VEC, true>(xe, carry, lane, xs);
#pragma unroll
    for (int m = 0; m < H2; ++m) {
      float2 gv = make_float2(de[m], de[m + H2]);
      if constexpr (SILU) {
        float2 s = make_float2(bv, bv);
#pragma unroll
        for (int w = 0; w < W; ++w) s = ffma2(make_float2(wv[w], wv[w]), make_float2(xs[m + w], xs[m + H2 + w]), s);
        if constexpr (HALF) gv = fmul2(gv, silu_grad_half_arg2_x2(s));
        else gv = fmul2(gv, silu_grad2(s));
      }
      g[m] = gv.x;
      g[m + H2] = gv.y;
    }
  };

  int left = n;
  bool started = false;  // the first row's values come from the prologue
  while (left > 0) {
    if (cc.step == 0 && started) {  // a new row: take the values loaded ahead
#pragma unroll
      for (int j = 0; j < W - 1; ++j) carry[j] = STATES ? ninit[j] : 0.f;
      if constexpr (STATES) {
        row_init<W>(a, row_after(a, cc), ninit);
        row_dfinal(cc);
      }
      if (cc.d != cur_d) {
        flush(cur_d);
#pragma unroll
        for (int w = 0; w < W; ++w) wv[w] = wn[w];
        bv = bn;
        cur_d = cc.d;
        channel_params<W>(a, cc.d + 1, sc, wn, bn);
      }
    }
    started = true;
    const int seg = min(static_cast<int>(a.nck) - cc.step, left);
    const bool row_ends = cc.step + seg == a.nck;
    int64_t pos = (int64_t)cc.step * S + lane * VEC;
    T* pdx = row_of<T>(a.dx, cc) + pos;
    float gprev[VEC];
#pragma unroll 2
    for (int k = 0; k < seg; ++k) {
      float xs[VEC + W - 1], g[VEC];
      next_g(xs, g);
      if (k > 0) {
        emit(pdx - S, pos - S, gprev, g, false);
      } else {  // the first step of the piece: seed the rotated right halo
#pragma unroll
        for (int j = 0; j < W - 1; ++j) rot_gs[j] = __shfl_sync(FULL, g[j], right);
      }
      // dinitial_states: dx at positions -(W-1) .. -1 of the row, from g at 0 .. W-2
      if (STATES && k == 0 && cc.step == 0 && a.dinit.data && lane == 0) {
#pragma unroll
        for (int kk = 0; kk < W - 1; ++kk) {
          float v = 0.f;
#pragma unroll
          for (int w = 0; w <= kk; ++w) v = fmaf(wv[w], g[kk - w], v);
          store_any(a.dinit.data, a.dinit.dtype, (int64_t)cc.b * a.dinit.s0 + (int64_t)cc.d * a.dinit.s1 + kk * a.dinit.s2, v);
        }
      }
#pragma unroll
      for (int m = 0; m < H2; ++m) {
        const float2 gm = make_float2(g[m], g[m + H2]);
        db = fadd2(db, gm);
#pragma unroll
        for (int w = 0; w < W; ++w) dw[w] = ffma2(gm, make_float2(xs[m + w], xs[m + H2 + w]), dw[w]);
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) gprev[i] = g[i];
      pos += S;
      pdx += S;
    }
    left -= seg;
    if (row_ends) {  // nothing right of the row's last step
      float zero[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) zero[i] = 0.f;
      emit(pdx - S, pos - S, gprev, zero, true);
      cc.step = 0;
      if (++cc.b == a.batch) {
        cc.b = 0;
        ++cc.d;
      }
    } else {  // the range ends inside the row: the right-halo step supplies g
      float xs[VEC + W - 1], g[VEC];
      next_g(xs, g);
      emit(pdx - S, pos - S, gprev, g, false);
      cc.step += seg;
    }
  }
  cp_async_wait<0>();
  flush(cur_d);
}

// Warp of the row walk that holds step q (inverse of part_start).
__device__ __forceinline__ int64_t walk_warp_of(int64_t q, int64_t nw, int64_t total) {
  const int64_t base = total / nw, rem = total - base * nw;
  const int64_t big = rem * (base + 1);
  return q < big ? q / (base + 1) : rem + (q - big) / base;
}

// dweight/dbias of channel d = the sum of its pieces in warp order.  One thread per
// (channel, value).
template <int W>
__global__ void __launch_bounds__(kThreads) reduce_rowwalk_partials(const ConvArgs a) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= a.dim * (W + 1)) return;
  grid_dependency_wait();  // the partials come from the kernel launched just before
  const int64_t d = t / (W + 1);
  const int k = static_cast<int>(t - d * (W + 1));
  const int64_t per = a.batch * a.nck;
  const int64_t w0 = walk_warp_of(d * per, a.ncol, a.units);
  const int64_t w1 = walk_warp_of((d + 1) * per - 1, a.ncol, a.units);
  float s = 0.f;
  for (int64_t w = w0; w <= w1; ++w) s += __ldcg(a.partials + (d + w) * (W + 1) + k);
  if (k < W) a.dweight[d * W + k] = s;
  else if (a.dbias) a.dbias[d] = s;
}

// ----------------------------------------------------------------- dispatch
template <typename T, int W>
static cudaError_t launch_rowwalk_w(bool bwd, const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  const bool states = bwd ? (a.init.data || a.dinit.data || a.dfinal.data) : (a.init.data || a.final_states.data);
#define CC1D_GO(K, SI, ST)                                                                   \
  {                                                                                          \
    const auto kern = K<T, W, SI, ST, kRowWalkDepth, kRowWalkThreads>;                       \
    const cudaError_t ea = allow_dynamic_smem(reinterpret_cast<const void*>(kern), ls.smem); \
    if (ea != cudaSuccess) return ea;                                                        \
    const cudaError_t el = launch_dependent(kern, ls.grid, dim3(kRowWalkThreads), ls.smem, s, a); \
    if (el != cudaSuccess) return el;                                                        \
  }
  if (!bwd) {
    if (ls.silu) { if (states) CC1D_GO(fwd_rowwalk_kernel, true, true) else CC1D_GO(fwd_rowwalk_kernel, true, false) }
    else { if (states) CC1D_GO(fwd_rowwalk_kernel, false, true) else CC1D_GO(fwd_rowwalk_kernel, false, false) }
    return cudaGetLastError();
  }
  if (ls.silu) { if (states) CC1D_GO(bwd_rowwalk_kernel, true, true) else CC1D_GO(bwd_rowwalk_kernel, true, false) }
  else { if (states) CC1D_GO(bwd_rowwalk_kernel, false, true) else CC1D_GO(bwd_rowwalk_kernel, false, false) }
#undef CC1D_GO
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((a.dim * (W + 1) + kThreads - 1) / kThreads));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, reduce_rowwalk_partials<W>, a);
}

cudaError_t CC1D_DT_NAME(rowwalk)(bool bwd, const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  switch (ls.width) {
    case 2: return launch_rowwalk_w<CC1D_DT_TYPE, 2>(bwd, a, ls, s);
    case 3: return launch_rowwalk_w<CC1D_DT_TYPE, 3>(bwd, a, ls, s);
    case 4: return launch_rowwalk_w<CC1D_DT_TYPE, 4>(bwd, a, ls, s);
    default: return cudaErrorInvalidValue;
  }
}

const void* CC1D_DT_NAME(rowwalk_kernel_ptr)(bool bwd, size_t smem) {
  const void* k = bwd ? reinterpret_cast<const void*>(bwd_rowwalk_kernel<CC1D_DT_TYPE, 4, true, false, kRowWalkDepth, kRowWalkThreads>)
                      : reinterpret_cast<const void*>(fwd_rowwalk_kernel<CC1D_DT_TYPE, 4, true, false, kRowWalkDepth, kRowWalkThreads>);
  allow_dynamic_smem(k, smem);  // so that the occupancy query sees the real limit
  return k;
}

}  // namespace cc1d
