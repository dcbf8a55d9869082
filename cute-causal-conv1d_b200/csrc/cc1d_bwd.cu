// Backward kernels of the depthwise causal conv1d (sm_100a).
//
// With p = bias + sum_w weight[w] * x[l-(W-1)+w] recomputed on the fly and
// g = dout * silu'(p) (or dout), one pass produces
//   dx[j]       = sum_k weight[W-1-k] * g[j+k]          (+ dfinal_states on the tail)
//   dweight[w] += g[l] * x[l-(W-1)+w],   dbias += g[l]
//   dinitial    = the dx formula at the W-1 positions before the sequence.
// seq_idx masks every tap whose two ends lie in different packed sequences.
//
// dweight / dbias are reduced deterministically: per-thread fp32 partials are summed
// in a fixed order inside the CTA, written to a per-tile slot of the workspace, and
// the last CTA to finish a channel tile (arrival counted with one atomicAdd, no
// waiting) sums the slots in slot order.  No float atomics anywhere, so results do
// not depend on scheduling.  Compiled once per element type (CC1D_DT).
#include "cc1d_common.cuh"
#include "cc1d_launch.h"

namespace cc1d {

template <int N, typename V>
__device__ __forceinline__ V pick_b(const V (&arr)[N], int idx) {
  V r = arr[0];
#pragma unroll
  for (int q = 1; q < N; ++q) r = (idx == q) ? arr[q] : r;
  return r;
}

// Sums the per-tile partials of one channel tile, in slot order, into dweight/dbias.
// `nslots` slots of `dim*(W+1)` floats; this CTA's tile covers channels
// [d_begin, d_begin + nch).
template <int W, int NT = kThreads>
__device__ __forceinline__ void reduce_tile_partials(const ConvArgs& a, int64_t nslots, int64_t d_begin,
                                                     int nch) {
  const int64_t row = a.dim * (W + 1);
  const int n = nch * (W + 1);
  for (int o = threadIdx.x; o < n; o += NT) {
    const int64_t d = d_begin + o / (W + 1);
    if (d >= a.dim) continue;
    const int w = o % (W + 1);
    const float* src = a.partials + d_begin * (W + 1) + o;
    // four independent chains, combined in a fixed order
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int64_t p = 0;
    for (; p + 4 <= nslots; p += 4) {
      s0 += __ldcg(src + (p + 0) * row);
      s1 += __ldcg(src + (p + 1) * row);
      s2 += __ldcg(src + (p + 2) * row);
      s3 += __ldcg(src + (p + 3) * row);
    }
    for (; p < nslots; ++p) s0 += __ldcg(src + p * row);
    const float s = (s0 + s1) + (s2 + s3);
    if (w < W) a.dweight[d * W + w] = s;
    else if (a.dbias) a.dbias[d] = s;
  }
}

// Arrival on a channel tile's counter; true in the CTA that arrived last.
__device__ __forceinline__ bool arrive_last(unsigned int* counter, unsigned int total) {
  __shared__ unsigned int s_ticket;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(counter, 1u);
  __syncthreads();
  const bool last = (s_ticket == total - 1);
  if (last) __threadfence();
  return last;
}

// ------------------------------------------------------------- channel-last
template <typename T, int W, int VEC, bool SILU, bool SEQ, int U>
__global__ void __launch_bounds__(kThreads) bwd_channel_last_kernel(const ConvArgs a) {
  extern __shared__ float red[];  // [kThreads * VEC * (W+1)]
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
    const bool active = cv < a.nv && l0 < L;
    const int64_t l1 = min(l0 + a.chunk, L);
    const int64_t d0 = cv * VEC;

    float dw[W][VEC], db[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      db[v] = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) dw[w][v] = 0.f;
    }

    if (active) {
      float wv[W][VEC], bv[VEC];
      load_params<W, VEC>(a, d0, wv, bv);
      const T* xrow = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 * a.x.s1;
      const T* grow = static_cast<const T*>(a.dout.data) + b * a.dout.s0 + d0 * a.dout.s1;
      T* dxrow = static_cast<T*>(a.dx.data) + b * a.dx.s0 + d0 * a.dx.s1;
      const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;

      float xw[W - 1][VEC], gw[W - 1][VEC];
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
#pragma unroll
        for (int v = 0; v < VEC; ++v) gw[k][v] = 0.f;
        if constexpr (SEQ) sw[k] = l >= 0 ? srow[l * a.seq_idx.s1] : -1;
      }
      const int64_t emit_lo = (l0 == 0 && a.dinit.data) ? -(int64_t)(W - 1) : l0;
      const int64_t lend = l1 + (W - 1);  // walk past the chunk to see g on the right halo
      const int64_t tail0 = L - (W - 1);  // first position fed by dfinal_states

      for (int64_t l = l0; l < lend; l += U) {
        Packet<T, VEC> rx[U], rg[U];
        int sq[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (l + u < L && l + u < lend) {
            rx[u] = ld_packet<T, VEC>(xrow + (l + u) * a.x.s2);
            rg[u] = ld_packet<T, VEC>(grow + (l + u) * a.dout.s2);
          }
          if constexpr (SEQ) sq[u] = (l + u < L && l + u < lend) ? srow[(l + u) * a.seq_idx.s1] : -1;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t ll = l + u;
          if (ll < lend) {
            const bool inside = ll < L;
            float xc[VEC], gc[VEC];
            if (inside) {
              unpack<T, VEC>(rx[u], xc);
              unpack<T, VEC>(rg[u], gc);
            } else {
#pragma unroll
              for (int v = 0; v < VEC; ++v) xc[v] = gc[v] = 0.f;
            }
            const int scur = SEQ ? sq[u] : 0;
            float g[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float gv = 0.f;
              if (inside) {
                if constexpr (SILU) {
                  float p = bv[v];
#pragma unroll
                  for (int w = 0; w < W - 1; ++w) {
                    float xin = xw[w][v];
                    if constexpr (SEQ) xin = (sw[w] == scur) ? xin : 0.f;
                    p = fmaf(wv[w][v], xin, p);
                  }
                  p = fmaf(wv[W - 1][v], xc[v], p);
                  if constexpr (SEQ) p = (scur >= 0) ? p : 0.f;
                  gv = gc[v] * silu_grad(p);
                } else {
                  gv = gc[v];
                }
                if constexpr (SEQ) gv = (scur >= 0) ? gv : 0.f;
              }
              g[v] = gv;
            }
            if (ll < l1) {
#pragma unroll
              for (int v = 0; v < VEC; ++v) {
                db[v] += g[v];
#pragma unroll
                for (int w = 0; w < W - 1; ++w) {
                  float xin = xw[w][v];
                  if constexpr (SEQ) xin = (sw[w] == scur) ? xin : 0.f;
                  dw[w][v] = fmaf(g[v], xin, dw[w][v]);
                }
                dw[W - 1][v] = fmaf(g[v], xc[v], dw[W - 1][v]);
              }
            }
            const int64_t e = ll - (W - 1);
            if (e >= emit_lo) {
              float dxv[VEC];
#pragma unroll
              for (int v = 0; v < VEC; ++v) {
                float s = 0.f;
#pragma unroll
                for (int k = 0; k < W - 1; ++k) {
                  float gk = gw[k][v];
                  if constexpr (SEQ) gk = (sw[0] == sw[k]) ? gk : 0.f;
                  s = fmaf(wv[W - 1 - k][v], gk, s);
                }
                {
                  float gk = g[v];
                  if constexpr (SEQ) gk = (sw[0] == scur) ? gk : 0.f;
                  s = fmaf(wv[0][v], gk, s);
                }
                if (a.dfinal.data && e >= tail0)
                  s += load_any(a.dfinal.data, a.dfinal.dtype,
                                b * a.dfinal.s0 + (d0 + v) * a.dfinal.s1 + (e - tail0) * a.dfinal.s2);
                dxv[v] = s;
              }
              if (e >= 0) {
                st_packet<T, VEC>(dxrow + e * a.dx.s2, pack<T, VEC>(dxv));
              } else {
#pragma unroll
                for (int v = 0; v < VEC; ++v)
                  store_any(a.dinit.data, a.dinit.dtype,
                            b * a.dinit.s0 + (d0 + v) * a.dinit.s1 + (e + W - 1) * a.dinit.s2, dxv[v]);
              }
            }
#pragma unroll
            for (int k = 0; k < W - 2; ++k) {
#pragma unroll
              for (int v = 0; v < VEC; ++v) {
                xw[k][v] = xw[k + 1][v];
                gw[k][v] = gw[k + 1][v];
              }
              if constexpr (SEQ) sw[k] = sw[k + 1];
            }
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              xw[W - 2][v] = xc[v];
              gw[W - 2][v] = g[v];
            }
            if constexpr (SEQ) sw[W - 2] = scur;
          }
        }
      }
    }

    // ---- deterministic dweight / dbias reduction
    float* mine = red + (size_t)threadIdx.x * VEC * (W + 1);
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
#pragma unroll
      for (int w = 0; w < W; ++w) mine[v * (W + 1) + w] = dw[w][v];
      mine[v * (W + 1) + W] = db[v];
    }
    __syncthreads();
    const int ncol = TX * VEC * (W + 1);  // floats per thread row (ty) in `red`
    const int64_t dbeg = bx * TX * VEC;
    const int64_t slot = b * a.nby + by;
    float* dst = a.partials + slot * a.dim * (W + 1) + dbeg * (W + 1);
    for (int o = threadIdx.x; o < ncol; o += kThreads) {
      float s = 0.f;
      for (int r = 0; r < TY; ++r) s += red[r * ncol + o];
      if (dbeg + o / (W + 1) < a.dim) dst[o] = s;
    }
    if (arrive_last(a.counters + bx, (unsigned)(a.nby * a.batch))) {
      reduce_tile_partials<W>(a, a.nby * a.batch, dbeg, TX * VEC);
      if (threadIdx.x == 0) a.counters[bx] = 0;  // leave the counter ready for the next launch
    }
    __syncthreads();  // `red` and the ticket are reused by the next tile
  }
}

// ----------------------------------------------------- channel-last, streamed
// Register state of one thread's walk down its row segment (VEC channels as H pairs).
template <typename T, int W, int VEC, bool SILU, bool SEQ>
struct BwdWalk {
  static constexpr int H = VEC / 2;
  // 16-bit tensors with SiLU: wv/bv hold weight/2 and bias/2, so the running sum is
  // h = p/2, g holds 2 * dout * silu'(p), dx = sum (w/2) g is exact, and the dweight /
  // dbias sums carry a factor 2 that is removed when they are stored.
  static constexpr bool HALF = SILU && sizeof(T) == 2;
  float2 wv[W][H], bv[H];
  float2 dw[W][H], db[H];
  float2 xw[W - 1][H], gw[W - 1][H];  // x and g at the W-1 rows before the current one
  int sw[W - 1];

  // One row: g = dout * silu'(p) at this row; optional dweight/dbias accumulation;
  // dx of the row W-1 earlier into `dxv`.  Windows advance by one row.  MASK applies the
  // seq_idx masks; a row whose window rows all carry its own non-negative seq_idx needs
  // none (every mask is 1).
  template <bool ACC, bool EMIT, bool MASK = SEQ>
  __device__ __forceinline__ void step(const float2 (&xc)[H], const float2 (&gc)[H], int scur, bool acc,
                                       float2 (&dxv)[H]) {
    float2 g[H];
#pragma unroll
    for (int i = 0; i < H; ++i) {
      float2 gv = gc[i];
      if constexpr (SILU) {
        float2 p = bv[i];
#pragma unroll
        for (int w = 0; w < W - 1; ++w) {
          float2 xin = xw[w][i];
          if constexpr (MASK) xin = (sw[w] == scur) ? xin : make_float2(0.f, 0.f);
          p = ffma2(wv[w][i], xin, p);
        }
        p = ffma2(wv[W - 1][i], xc[i], p);
        if constexpr (MASK) p = (scur >= 0) ? p : make_float2(0.f, 0.f);
        if constexpr (HALF) gv = fmul2(gv, silu_grad_half_arg2_x2(p));
        else gv = fmul2(gv, silu_grad2(p));
      }
      if constexpr (MASK) gv = (scur >= 0) ? gv : make_float2(0.f, 0.f);
      g[i] = gv;
    }
    if (ACC && acc) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        db[i] = fadd2(db[i], g[i]);
#pragma unroll
        for (int w = 0; w < W - 1; ++w) {
          float2 xin = xw[w][i];
          if constexpr (MASK) xin = (sw[w] == scur) ? xin : make_float2(0.f, 0.f);
          dw[w][i] = ffma2(g[i], xin, dw[w][i]);
        }
        dw[W - 1][i] = ffma2(g[i], xc[i], dw[W - 1][i]);
      }
    }
    if constexpr (EMIT) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float2 s = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < W - 1; ++k) {
          float2 gk = gw[k][i];
          if constexpr (MASK) gk = (sw[0] == sw[k]) ? gk : make_float2(0.f, 0.f);
          s = ffma2(wv[W - 1 - k][i], gk, s);
        }
        float2 gk = g[i];
        if constexpr (MASK) gk = (sw[0] == scur) ? gk : make_float2(0.f, 0.f);
        dxv[i] = ffma2(wv[0][i], gk, s);
      }
    }
#pragma unroll
    for (int k = 0; k < W - 2; ++k) {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        xw[k][i] = xw[k + 1][i];
        gw[k][i] = gw[k + 1][i];
      }
      sw[k] = sw[k + 1];
    }
#pragma unroll
    for (int i = 0; i < H; ++i) {
      xw[W - 2][i] = xc[i];
      gw[W - 2][i] = g[i];
    }
    sw[W - 2] = scur;
  }
};

// One wave of persistent warps (see WarpUnit), one CTA of NT = 512 threads per SM (one
// CTA of 16 warps keeps the warps' progress closer together than four CTAs of 4, whose
// warps the scheduler serves by CTA age): lane = one VEC-channel packet, warp =
// 32 consecutive packets of one batch row and one segment [l0, l1).  The x rows l0-(W-1) .. l0-1 (or initial states)
// are read once into the window; x and dout rows l0 .. l1+W-2 stream through private
// cp.async rings (zero filled past L, so g vanishes there without a check).  Row l
// produces g[l] (dweight/dbias terms when l < l1) and dx[l-(W-1)].  The first W-1 rows
// (dinitial_states) and the W-1 rows past l1 (dfinal_states) take a checked path; the
// rows between run unrolled blocks of P rows with compile-time ring slots, predicated
// prefetch and no branches.
template <typename T, int W, int VEC, bool SILU, bool SEQ, int P, int NT>
__global__ void __launch_bounds__(NT) bwd_stream_kernel(const ConvArgs a) {
  grid_dependency_wait();  // launched as a programmatic dependent launch
  using Pk = Packet<T, VEC>;
  constexpr int H = VEC / 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Pk* xring = reinterpret_cast<Pk*>(smem_raw) + threadIdx.x;
  Pk* gring = reinterpret_cast<Pk*>(smem_raw) + P * NT + threadIdx.x;
  const int lane = threadIdx.x & 31;
  // warps take units round robin over the CTAs, so that fewer units than resident warps
  // still spread over every SM (the host sizes the grid)
  const int64_t unit = (int64_t)(threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  if (unit >= a.units) return;  // whole warps only
  const WarpUnit wu = warp_unit(a, unit);
  const int64_t pb = static_cast<unsigned>(wu.col) / static_cast<unsigned>(a.batch);  // packet block
  const int64_t b = wu.col - pb * a.batch;
  const int64_t cv = pb * 32 + lane;
  const int64_t L = a.seqlen;
  const int64_t l0 = part_start(wu.seg, wu.nseg, L);
  const int64_t l1_seg = part_start(wu.seg + 1, wu.nseg, L);
  const bool active = cv < a.nv && l0 < l1_seg;
  const int64_t d0 = cv * VEC;

  BwdWalk<T, W, VEC, SILU, SEQ> st;
#pragma unroll
  for (int i = 0; i < H; ++i) {
    st.db[i] = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < W; ++w) st.dw[w][i] = make_float2(0.f, 0.f);
  }

  if (active) {
    const int64_t l1 = l1_seg;
    const int nmain = static_cast<int>(l1 - l0);                   // rows that accumulate
    const int nload = static_cast<int>(min(l1 + (W - 1), L) - l0);  // rows with data
    const int nall = nmain + (W - 1);                                // rows walked
    const int64_t sx = a.x.s2, sg = a.dout.s2, sd = a.dx.s2;
    const T* xsrc = static_cast<const T*>(a.x.data) + b * a.x.s0 + d0 + l0 * sx;
    const T* gsrc = static_cast<const T*>(a.dout.data) + b * a.dout.s0 + d0 + l0 * sg;
    // stream row j <-> position l0 + j, ring slot j % P; rows past the data are zero filled
#pragma unroll
    for (int j = 0; j < P - 1; ++j) {
      cp_async_packet<sizeof(Pk)>(xring + j * NT, xsrc, j < nload);
      cp_async_packet<sizeof(Pk)>(gring + j * NT, gsrc, j < nload);
      xsrc += sx;
      gsrc += sg;
      cp_async_commit();
    }

    // parameter and window loads are all issued before the first use of either
    {
      float wf[W][VEC], bf[VEC];
      load_params<W, VEC>(a, d0, wf, bf);
      load_window<T, W, VEC>(a, b, d0, l0, st.xw);
      constexpr float k = decltype(st)::HALF ? 0.5f : 1.0f;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        st.bv[i] = make_float2(k * bf[2 * i], k * bf[2 * i + 1]);
#pragma unroll
        for (int w = 0; w < W; ++w) st.wv[w][i] = make_float2(k * wf[w][2 * i], k * wf[w][2 * i + 1]);
      }
    }
    const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
      const int64_t l = l0 - (W - 1) + k;
#pragma unroll
      for (int i = 0; i < H; ++i) st.gw[k][i] = make_float2(0.f, 0.f);
      st.sw[k] = (SEQ && l >= 0) ? srow[l * a.seq_idx.s1] : -1;
    }
    const int64_t tail0 = L - (W - 1);
    // row j emits dx at e = l0 + j - (W-1): rows j >= W-1 of every segment, plus the first
    // W-1 rows of the first segment when dinitial_states are wanted (e < 0)
    const int emit0 = (l0 == 0 && a.dinit.data != nullptr) ? 0 : W - 1;
    T* dxptr = static_cast<T*>(a.dx.data) + b * a.dx.s0 + d0 + (l0 - (W - 1)) * sd;

    // Rows with a rare case: accumulation stops at nmain, dx of position
    // e = l0 + j - (W-1) goes to dinitial_states (e < 0) or gets dfinal_states (e >= L-(W-1)).
    auto generic_row = [&](int j, const Pk& rx, const Pk& rg) {
      float2 xc[H], gc[H];
      unpack2<T, VEC>(rx, xc);
      unpack2<T, VEC>(rg, gc);
      int scur = 0;
      if constexpr (SEQ) scur = j < nload ? srow[(l0 + j) * a.seq_idx.s1] : -1;
      float2 dxv[H];
      st.template step<true, true>(xc, gc, scur, j < nmain, dxv);
      if (j >= emit0) {
        const int64_t e = l0 + j - (W - 1);
        if (a.dfinal.data && e >= tail0) {
#pragma unroll
          for (int i = 0; i < H; ++i) {
            const int64_t o = b * a.dfinal.s0 + (d0 + 2 * i) * a.dfinal.s1 + (e - tail0) * a.dfinal.s2;
            dxv[i].x += load_any(a.dfinal.data, a.dfinal.dtype, o);
            dxv[i].y += load_any(a.dfinal.data, a.dfinal.dtype, o + a.dfinal.s1);
          }
        }
        if (e >= 0) {
          st_packet<T, VEC>(dxptr, pack2<T, VEC>(dxv));
        } else {
#pragma unroll
          for (int i = 0; i < H; ++i) {
            const int64_t o = b * a.dinit.s0 + (d0 + 2 * i) * a.dinit.s1 + (e + W - 1) * a.dinit.s2;
            store_any(a.dinit.data, a.dinit.dtype, o, dxv[i].x);
            store_any(a.dinit.data, a.dinit.dtype, o + a.dinit.s1, dxv[i].y);
          }
        }
      }
      dxptr += sd;
    };
    // Steady rows (W-1 <= j < nmain): accumulate, emit dx at e >= l0, nothing rare.
    const int* sptr = SEQ ? srow + (l0 + W - 1) * a.seq_idx.s1 : nullptr;
    auto steady_row = [&](const Pk& rx, const Pk& rg) {
      float2 xc[H], gc[H];
      unpack2<T, VEC>(rx, xc);
      unpack2<T, VEC>(rg, gc);
      int scur = 0;
      if constexpr (SEQ) {
        scur = *sptr;
        sptr += a.seq_idx.s1;
      }
      float2 dxv[H];
      st.template step<true, true>(xc, gc, scur, true, dxv);
      st_packet<T, VEC>(dxptr, pack2<T, VEC>(dxv));
      dxptr += sd;
    };
    auto prefetch = [&](int j, int slot) {  // row j + P - 1 into `slot`
      const bool ok = j + P - 1 < nload;
      cp_async_packet<sizeof(Pk)>(xring + slot * NT, xsrc, ok);
      cp_async_packet<sizeof(Pk)>(gring + slot * NT, gsrc, ok);
      xsrc += sx;
      gsrc += sg;
      cp_async_commit();
      cp_async_wait<P - 1>();
    };
    // head: rows 0 .. W-2
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      if (j < nall) {
        prefetch(j, (j + P - 1) % P);
        generic_row(j, xring[j * NT], gring[j * NT]);
      }
    }
    // steady: rows W-1 .. nmain-1 in unrolled blocks of P (compile-time slots), then the rest
    int j = W - 1;
    bool plain_blocks = true;
    if constexpr (SEQ) {
      // Warps whose 32 lanes all hold channels read the seq_idx of 32 steady rows at a
      // time, one per lane (steady row W-1 + r in lane r % 32 of chunk r / 32), the next
      // chunk one chunk ahead.  A block whose P rows and W-1 window rows all carry one
      // non-negative id runs the step without masks; any other block goes row by row
      // with the masks.  The result is the same either way.
      if (pb * 32 + 32 <= a.nv) {
        plain_blocks = false;
        constexpr unsigned FULL = 0xffffffffu;
        const int* ids = srow + (l0 + W - 1) * a.seq_idx.s1;
        const int nsteady = nmain - (W - 1);
        auto load_ids = [&](int r0) {
          const int r = r0 + lane;
          return r < nsteady ? __ldg(ids + static_cast<int64_t>(r) * a.seq_idx.s1) : -1;
        };
        int cur = load_ids(0), nxt = load_ids(32);
        int k = 0;  // first row of the block within the chunk
        for (; j + P <= nmain; j += P) {
          const int v = st.sw[0];
          bool same = v >= 0;
#pragma unroll
          for (int w = 1; w < W - 1; ++w) same = same && st.sw[w] == v;
          same = __all_sync(FULL, same && (static_cast<unsigned>(lane - k) >= static_cast<unsigned>(P) || cur == v));
          if (same) {
#pragma unroll
            for (int u = 0; u < P; ++u) {
              prefetch(j + u, (u + W - 1 + P - 1) % P);
              const Pk& rx = xring[((u + W - 1) % P) * NT];
              const Pk& rg = gring[((u + W - 1) % P) * NT];
              float2 xc[H], gc[H];
              unpack2<T, VEC>(rx, xc);
              unpack2<T, VEC>(rg, gc);
              float2 dxv[H];
              st.template step<true, true, false>(xc, gc, v, true, dxv);
              st_packet<T, VEC>(dxptr, pack2<T, VEC>(dxv));
              dxptr += sd;
            }
            sptr += P * a.seq_idx.s1;
          } else {
            for (int u = 0; u < P; ++u) {  // rare: row by row, reading each row's id
              prefetch(j + u, (j + u + P - 1) % P);
              steady_row(xring[((j + u) % P) * NT], gring[((j + u) % P) * NT]);
            }
          }
          k += P;
          if (k == 32) {
            k = 0;
            cur = nxt;
            nxt = load_ids(j + P - (W - 1) + 32);
          }
        }
      }
    }
    if (plain_blocks) {
      for (; j + P <= nmain; j += P) {
#pragma unroll
        for (int u = 0; u < P; ++u) {
          prefetch(j + u, (u + W - 1 + P - 1) % P);
          steady_row(xring[((u + W - 1) % P) * NT], gring[((u + W - 1) % P) * NT]);
        }
      }
    }
    for (; j < nmain; ++j) {
      prefetch(j, (j + P - 1) % P);
      steady_row(xring[(j % P) * NT], gring[(j % P) * NT]);
    }
    // tail: rows max(W-1, nmain) .. nall-1 (no accumulation; dfinal_states; zeros past L)
    for (j = max(W - 1, nmain); j < nall; ++j) {
      prefetch(j, (j + P - 1) % P);
      generic_row(j, xring[(j % P) * NT], gring[(j % P) * NT]);
    }
  }
  cp_async_wait<0>();

  // ---- dweight / dbias: each warp unit writes its partial sums to its own slot; the
  // next kernel (reduce_unit_partials) adds the slots of each channel in unit order.
  // The unit's slab is value-major ([VEC * (W + 1)][32 lanes]): each store below writes
  // one 128-byte line.
  constexpr int PER_LANE = VEC * (W + 1);
  constexpr float k = decltype(st)::HALF ? 0.5f : 1.0f;  // exact
  float* mine = a.partials + unit * 32 * PER_LANE + lane;
#pragma unroll
  for (int i = 0; i < H; ++i) {
#pragma unroll
    for (int w = 0; w < W; ++w) {
      mine[((2 * i) * (W + 1) + w) * 32] = k * st.dw[w][i].x;
      mine[((2 * i + 1) * (W + 1) + w) * 32] = k * st.dw[w][i].y;
    }
    mine[((2 * i) * (W + 1) + W) * 32] = k * st.db[i].x;
    mine[((2 * i + 1) * (W + 1) + W) * 32] = k * st.db[i].y;
  }
}

// Deterministic sum of the warp-unit partials of the streamed backward kernels.  Slot
// layout [unit][PER_LANE][32 lanes]; lane l of packet block pb covers channels
// (pb*32 + l)*VEC .. +VEC-1 and PER_LANE = VEC*(W+1) values (W weights, then bias, per
// channel), so one unit's slots form a contiguous slab of 32*PER_LANE floats, and the
// units of packet block pb (all batch rows, all segments) are contiguous.
// A block owns one value index r of one packet block (32 lanes); each of its
// kReduceChains warps adds every kReduceChains-th unit in unit order (loads issued
// sixteen at a time), and warp 0 adds the chains in chain order.  The order of every addition
// depends only on the geometry, so the result is reproducible.
constexpr int kReduceChains = 8;

template <int W, int VEC>
__global__ void __launch_bounds__(32 * kReduceChains) reduce_unit_partials(const ConvArgs a) {
  constexpr int PER_LANE = VEC * (W + 1);
  constexpr int64_t SLAB = 32 * PER_LANE;
  constexpr int S = kReduceChains;
  __shared__ float chain_sum[S][32];
  const int lane = threadIdx.x & 31;
  const int chain = threadIdx.x >> 5;
  const int64_t pb = blockIdx.x / PER_LANE;
  const int r = static_cast<int>(blockIdx.x % PER_LANE);  // value index
  const int q = r * 32 + lane;                            // slab position
  grid_dependency_wait();  // the partials come from the kernel launched just before
  const int64_t u0 = first_unit(a, pb * a.batch), u1 = first_unit(a, (pb + 1) * a.batch);
  const float* src = a.partials + q;
  float acc = 0.f;
  // up to 16 units per chain are loaded at once (one L2 round trip for up to 128 units
  // per packet block), then added in unit order
  constexpr int BATCH = 16;
  for (int64_t k = u0 + chain; k < u1; k += BATCH * S) {
    float v[BATCH];
#pragma unroll
    for (int i = 0; i < BATCH; ++i) v[i] = (k + i * S < u1) ? __ldcg(src + (k + i * S) * SLAB) : 0.f;
#pragma unroll
    for (int i = 0; i < BATCH; ++i)
      if (k + i * S < u1) acc += v[i];
  }
  chain_sum[chain][lane] = acc;
  __syncthreads();
  if (chain != 0) return;
  float sum = chain_sum[0][lane];
#pragma unroll
  for (int c = 1; c < S; ++c) sum += chain_sum[c][lane];
  const int64_t d = (pb * 32 + lane) * VEC + r / (W + 1);
  const int w = r % (W + 1);
  if (d >= a.dim) return;
  if (w < W) a.dweight[d * W + w] = sum;
  else if (a.dbias) a.dbias[d] = sum;
}

// Launches reduce_unit_partials right behind the kernel that wrote the partials, as a
// programmatic dependent launch: its blocks are scheduled as the writer's blocks retire
// and wait in grid_dependency_wait() for the writer's results.
template <int W, int VEC>
static cudaError_t launch_reduce(const ConvArgs& a, cudaStream_t s) {
  constexpr int PER_LANE = VEC * (W + 1);
  const int64_t npb = (a.nv + 31) / 32;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(npb * PER_LANE));
  cfg.blockDim = dim3(32 * kReduceChains);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, reduce_unit_partials<W, VEC>, a);
}

// ------------------------------------------------------------------- rows
template <typename T, int W, int VEC, bool SILU, bool SEQ>
__global__ void __launch_bounds__(kThreads) bwd_row_kernel(const ConvArgs a) {
  constexpr unsigned FULL = 0xffffffffu;
  const int G = 1 << a.g_shift;
  const int gl = threadIdx.x & (G - 1);
  const int group = threadIdx.x >> a.g_shift;
  const int DPB = kThreads >> a.g_shift;
  const int64_t L = a.seqlen;
  const int64_t span = (int64_t)G * VEC;
  const int64_t ntiles = a.nbx * a.nck * a.batch;
  const int64_t tail0 = L - (W - 1);

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
    const T* grow = static_cast<const T*>(a.dout.data) + b * a.dout.s0 + dd * a.dout.s1;
    T* dxrow = static_cast<T*>(a.dx.data) + b * a.dx.s0 + dd * a.dx.s1;
    const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;

    float wv[W], bias;
    {
      float wt[W][1], bt[1];
      load_params<W, 1>(a, dd, wt, bt);
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w] = wt[w][0];
      bias = bt[0];
    }

    float carry[W - 1];
    int scarry[W - 1];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const int64_t pos = cs - (W - 1) + j;
      float v = 0.f;
      if (row_ok) {
        if (pos >= 0) v = to_f32(xrow[pos]);
        else if (a.init.data)
          v = load_any(a.init.data, a.init.dtype, b * a.init.s0 + dd * a.init.s1 + (W - 1 + pos) * a.init.s2);
      }
      carry[j] = v;
      if constexpr (SEQ) scarry[j] = (row_ok && pos >= 0) ? srow[pos * a.seq_idx.s1] : -1;
    }

    float gprev[VEC];
    int sprev[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      gprev[i] = 0.f;
      sprev[i] = -1;
    }
    float dw[W], db = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) dw[w] = 0.f;

    for (int r = 0; r <= a.rounds; ++r) {
      const int64_t rs = cs + r * span;
      const int64_t e0 = rs + gl * VEC;
      // the last pass only looks at the W-1 positions right of the chunk
      const int64_t lim = (r < a.rounds) ? ce : min(L, ce + (W - 1));
      float xv[VEC], gv[VEC];
      int sv[VEC];
      if (row_ok && e0 + VEC <= lim) {
        unpack<T, VEC>(ld_packet<T, VEC>(xrow + e0), xv);
        unpack<T, VEC>(ld_packet<T, VEC>(grow + e0), gv);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const bool ok = row_ok && e0 + i < lim;
          xv[i] = ok ? to_f32(xrow[e0 + i]) : 0.f;
          gv[i] = ok ? to_f32(grow[e0 + i]) : 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        if constexpr (SEQ) sv[i] = (row_ok && e0 + i < lim) ? srow[(e0 + i) * a.seq_idx.s1] : -1;
        else sv[i] = 0;
      }

      // x (and seq_idx) from e0-(W-1) to e0+VEC-1
      float xs[VEC + W - 1];
      int ss[VEC + W - 1];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        xs[W - 1 + i] = xv[i];
        ss[W - 1 + i] = sv[i];
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
          hv = pick_b<W - 1>(carry, idx);
          if constexpr (SEQ) hs = pick_b<W - 1>(scarry, idx);
        }
        xs[W - 1 - k] = hv;
        ss[W - 1 - k] = hs;
      }

      float g[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        float gg = gv[i];
        if constexpr (SILU) {
          float p = bias;
#pragma unroll
          for (int w = 0; w < W; ++w) {
            float xin = xs[i + w];
            if constexpr (SEQ) xin = (ss[i + w] == ss[W - 1 + i]) ? xin : 0.f;
            p = fmaf(wv[w], xin, p);
          }
          if constexpr (SEQ) p = (ss[W - 1 + i] >= 0) ? p : 0.f;
          gg = gg * silu_grad(p);
        }
        if constexpr (SEQ) gg = (ss[W - 1 + i] >= 0) ? gg : 0.f;
        g[i] = (row_ok && e0 + i < lim) ? gg : 0.f;
      }

      if (r < a.rounds) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          db += g[i];
#pragma unroll
          for (int w = 0; w < W; ++w) {
            float xin = xs[i + w];
            if constexpr (SEQ) xin = (ss[i + w] == ss[W - 1 + i]) ? xin : 0.f;
            dw[w] = fmaf(g[i], xin, dw[w]);
          }
        }
      }

      // dinitial_states: the dx formula at positions -(W-1)..-1 of the first chunk
      if (r == 0 && c == 0 && a.dinit.data) {
        float gh[W - 1];
#pragma unroll
        for (int q = 0; q < W - 1; ++q) gh[q] = __shfl_sync(FULL, g[q % VEC], q / VEC, G);
        if (row_ok && gl == 0) {
#pragma unroll
          for (int j = 0; j < W - 1; ++j) {
            const int64_t pos = j - (W - 1);
            float s = 0.f;
            if constexpr (!SEQ) {
#pragma unroll
              for (int k = 0; k < W; ++k) {
                const int q = j - (W - 1) + k;  // position of g
                if (q >= 0) s = fmaf(wv[W - 1 - k], gh[q], s);
              }
            }
            if (a.dfinal.data && pos >= tail0)
              s += load_any(a.dfinal.data, a.dfinal.dtype, b * a.dfinal.s0 + d * a.dfinal.s1 + (pos - tail0) * a.dfinal.s2);
            store_any(a.dinit.data, a.dinit.dtype, b * a.dinit.s0 + d * a.dinit.s1 + j * a.dinit.s2, s);
          }
        }
      }

      // dx for the previous round's positions: needs g of the W-1 positions after each
      if (r > 0) {
        float gx[VEC + W - 1];
        int sx[VEC + W - 1];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          gx[i] = gprev[i];
          sx[i] = sprev[i];
        }
#pragma unroll
        for (int q = 0; q < W - 1; ++q) {
          const int delta = 1 + q / VEC;
          const int slot = q % VEC;
          const float va = __shfl_down_sync(FULL, gprev[slot], delta, G);
          const int src = (gl + delta - G) & (G - 1);
          const float vb = __shfl_sync(FULL, g[slot], src, G);
          gx[VEC + q] = (gl + delta < G) ? va : vb;
          if constexpr (SEQ) {
            const int sa = __shfl_down_sync(FULL, sprev[slot], delta, G);
            const int sb = __shfl_sync(FULL, sv[slot], src, G);
            sx[VEC + q] = (gl + delta < G) ? sa : sb;
          }
        }
        const int64_t p0 = rs - span + gl * VEC;  // first position of this lane's previous packet
        float dxv[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          float s = 0.f;
#pragma unroll
          for (int k = 0; k < W; ++k) {
            float gk = gx[i + k];
            if constexpr (SEQ) gk = (sx[i] == sx[i + k]) ? gk : 0.f;
            s = fmaf(wv[W - 1 - k], gk, s);
          }
          const int64_t e = p0 + i;
          if (a.dfinal.data && e >= tail0 && e < L && row_ok)
            s += load_any(a.dfinal.data, a.dfinal.dtype, b * a.dfinal.s0 + d * a.dfinal.s1 + (e - tail0) * a.dfinal.s2);
          dxv[i] = s;
        }
        if (row_ok && p0 + VEC <= ce) {
          st_packet<T, VEC>(dxrow + p0, pack<T, VEC>(dxv));
        } else if (row_ok) {
#pragma unroll
          for (int i = 0; i < VEC; ++i)
            if (p0 + i < ce) dxrow[p0 + i] = from_f32<T>(dxv[i]);
        }
      }

#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        gprev[i] = g[i];
        sprev[i] = sv[i];
      }
#pragma unroll
      for (int j = 0; j < W - 1; ++j) {
        const int m = W - 1 - j;
        const int delta = (m + VEC - 1) / VEC;
        const int slot = delta * VEC - m;
        carry[j] = __shfl_sync(FULL, xv[slot], G - delta, G);
        if constexpr (SEQ) scarry[j] = __shfl_sync(FULL, sv[slot], G - delta, G);
      }
    }

    // ---- deterministic reduction: group butterfly, then per-tile slot, then last CTA
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      if (off < G) {
#pragma unroll
        for (int w = 0; w < W; ++w) dw[w] += __shfl_xor_sync(FULL, dw[w], off, G);
        db += __shfl_xor_sync(FULL, db, off, G);
      }
    }
    const int64_t slot = b * a.nck + c;
    if (row_ok && gl == 0) {
      float* dst = a.partials + slot * a.dim * (W + 1) + d * (W + 1);
#pragma unroll
      for (int w = 0; w < W; ++w) dst[w] = dw[w];
      dst[W] = db;
    }
    if (arrive_last(a.counters + dtile, (unsigned)(a.nck * a.batch))) {
      reduce_tile_partials<W>(a, a.nck * a.batch, dtile * DPB, DPB);
      if (threadIdx.x == 0) a.counters[dtile] = 0;
    }
    __syncthreads();
  }
}

// ----------------------------------------------------------------- dispatch
template <typename T, int W, int VEC>
static cudaError_t launch_bwd_w(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  const bool silu = ls.silu, seq = ls.seq;
  if (ls.layout == kLayoutStream) {
    if constexpr (VEC * sizeof(T) == kBwdPacketBytes) {
#define CC1D_GO(SI, SQ)                                                                               \
  {                                                                                                   \
    const auto kern = bwd_stream_kernel<T, W, VEC, SI, SQ, kStreamDepth, kBwdStreamThreads>;           \
    const cudaError_t ea = allow_dynamic_smem(reinterpret_cast<const void*>(kern), ls.smem);                   \
    if (ea != cudaSuccess) return ea;                                                                 \
    const cudaError_t el = launch_dependent(kern, ls.grid, dim3(kBwdStreamThreads), ls.smem, s, a);    \
    if (el != cudaSuccess) return el;                                                                 \
  }
      if (silu) { if (seq) CC1D_GO(true, true) else CC1D_GO(true, false) }
      else { if (seq) CC1D_GO(false, true) else CC1D_GO(false, false) }
#undef CC1D_GO
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      return launch_reduce<W, VEC>(a, s);
    }
  } else if (ls.layout == kLayoutChannelLast) {
    constexpr int U = 2;
#define CC1D_GO(SI, SQ) bwd_channel_last_kernel<T, W, VEC, SI, SQ, U><<<ls.grid, kThreads, ls.smem, s>>>(a)
    if (silu) { if (seq) CC1D_GO(true, true); else CC1D_GO(true, false); }
    else { if (seq) CC1D_GO(false, true); else CC1D_GO(false, false); }
#undef CC1D_GO
  } else {
#define CC1D_GO(SI, SQ) bwd_row_kernel<T, W, VEC, SI, SQ><<<ls.grid, kThreads, 0, s>>>(a)
    if (silu) { if (seq) CC1D_GO(true, true); else CC1D_GO(true, false); }
    else { if (seq) CC1D_GO(false, true); else CC1D_GO(false, false); }
#undef CC1D_GO
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_bwd_t(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  constexpr int PV = 16 / sizeof(T);
  constexpr int SV = kBwdPacketBytes / sizeof(T);  // the streamed kernel's packets
  if (ls.layout == kLayoutStream) {
    switch (ls.width) {
      case 2: return launch_bwd_w<T, 2, SV>(a, ls, s);
      case 3: return launch_bwd_w<T, 3, SV>(a, ls, s);
      case 4: return launch_bwd_w<T, 4, SV>(a, ls, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (ls.width * 2 + (ls.packet ? 1 : 0)) {
    case 4: return launch_bwd_w<T, 2, 1>(a, ls, s);
    case 5: return launch_bwd_w<T, 2, PV>(a, ls, s);
    case 6: return launch_bwd_w<T, 3, 1>(a, ls, s);
    case 7: return launch_bwd_w<T, 3, PV>(a, ls, s);
    case 8: return launch_bwd_w<T, 4, 1>(a, ls, s);
    case 9: return launch_bwd_w<T, 4, PV>(a, ls, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static const void* bwd_kernel_ptr_t(const LaunchShape& ls) {
  constexpr int PV = 16 / sizeof(T);
  if (ls.layout == kLayoutStream) {
    const void* k = reinterpret_cast<const void*>(
        bwd_stream_kernel<T, 4, kBwdPacketBytes / sizeof(T), true, false, kStreamDepth, kBwdStreamThreads>);
    allow_dynamic_smem(k, ls.smem);  // so that the occupancy query sees the real limit
    return k;
  }
  if (ls.layout == kLayoutChannelLast) {
    if (ls.packet) return reinterpret_cast<const void*>(bwd_channel_last_kernel<T, 4, PV, true, false, 2>);
    return reinterpret_cast<const void*>(bwd_channel_last_kernel<T, 4, 1, true, false, 2>);
  }
  if (ls.packet) return reinterpret_cast<const void*>(bwd_row_kernel<T, 4, PV, true, false>);
  return reinterpret_cast<const void*>(bwd_row_kernel<T, 4, 1, true, false>);
}

cudaError_t CC1D_DT_NAME(bwd)(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  return launch_bwd_t<CC1D_DT_TYPE>(a, ls, s);
}

// Sum of the row-stream kernel's warp-unit partials (one channel per lane: VEC = 1).
cudaError_t CC1D_DT_NAME(reduce_rows)(const ConvArgs& a, int width, cudaStream_t s) {
  switch (width) {
    case 2: return launch_reduce<2, 1>(a, s);
    case 3: return launch_reduce<3, 1>(a, s);
    case 4: return launch_reduce<4, 1>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

const void* CC1D_DT_NAME(bwd_kernel_ptr)(const LaunchShape& ls) {
  return bwd_kernel_ptr_t<CC1D_DT_TYPE>(ls);
}

}  // namespace cc1d
