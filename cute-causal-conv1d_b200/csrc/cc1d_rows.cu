// Streamed backward kernel for (batch, dim, seqlen)-contiguous tensors (sm_100a).
//
// Lane = one channel row, warp = 32 consecutive channels of one batch row and one
// sequence segment (the WarpUnit split of cc1d_common.cuh).  Each step moves C positions
// of the lane's row (one 32-byte sector: 16 positions of a 16-bit type, 8 of fp32)
// through a private ring of P shared-memory slots filled with cp.async, so P-1 sectors
// per lane are in flight without registers.  The W-1 element window and (backward)
// the g values of the previous step stay in registers: no halo is re-read and no lane
// exchanges data.  Every sector of the row is read exactly once; stores are aligned
// 16-byte pairs.  Compiled once per element type (CC1D_DT).
#include "cc1d_common.cuh"
#include "cc1d_launch.h"

namespace cc1d {

template <typename T>
struct RowStep {
  static constexpr int C = 32 / sizeof(T);  // positions per step (one 32-byte sector)
  uint4 q[2];
};

template <typename T>
__device__ __forceinline__ void step_to_f32(const RowStep<T>& r, float (&f)[RowStep<T>::C]) {
  constexpr int C = RowStep<T>::C;
  const unsigned* u = reinterpret_cast<const unsigned*>(&r);
  if constexpr (std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < C; ++i) f[i] = __uint_as_float(u[i]);
  } else if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
  }
}

template <typename T>
__device__ __forceinline__ RowStep<T> f32_to_step(const float (&f)[RowStep<T>::C]) {
  constexpr int C = RowStep<T>::C;
  RowStep<T> r;
  unsigned* u = reinterpret_cast<unsigned*>(&r);
  if constexpr (std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < C; ++i) u[i] = __float_as_uint(f[i]);
  } else if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      u[i] = *reinterpret_cast<unsigned*>(&h);
    }
  } else {
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      u[i] = *reinterpret_cast<unsigned*>(&h);
    }
  }
  return r;
}

// Copy `count` (0..C) positions starting at `src` into a ring slot; the rest is zero.
template <typename T>
__device__ __forceinline__ void issue_step(RowStep<T>* slot, const T* src, int count) {
  const int bytes = count * static_cast<int>(sizeof(T));
  const int b0 = bytes < 16 ? bytes : 16;
  const int b1 = bytes > 16 ? bytes - 16 : 0;
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(slot));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(src), "r"(b0) : "memory");
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s + 16), "l"(b1 ? src + 16 / sizeof(T) : src),
               "r"(b1)
               : "memory");
}

template <typename T>
__device__ __forceinline__ void store_step(T* dst, const RowStep<T>& r, int count) {
  constexpr int C = RowStep<T>::C;
  if (count == C) {
    reinterpret_cast<uint4*>(dst)[0] = r.q[0];
    reinterpret_cast<uint4*>(dst)[1] = r.q[1];
  } else {
    const T* v = reinterpret_cast<const T*>(&r);
    for (int i = 0; i < count; ++i) dst[i] = v[i];
  }
}

// Lane geometry shared by both kernels.
struct RowLane {
  int64_t b, d, pb, l0, l1;
  bool active;
};
template <int C>
__device__ __forceinline__ RowLane row_lane(const ConvArgs& a, int64_t unit, int lane) {
  const WarpUnit wu = warp_unit(a, unit);
  RowLane r;
  r.pb = static_cast<unsigned>(wu.col) / static_cast<unsigned>(a.batch);
  r.b = wu.col - r.pb * a.batch;
  r.d = r.pb * 32 + lane;
  const int64_t nsteps = (a.seqlen + C - 1) / C;
  r.l0 = min(a.seqlen, part_start(wu.seg, wu.nseg, nsteps) * C);
  r.l1 = min(a.seqlen, part_start(wu.seg + 1, wu.nseg, nsteps) * C);
  r.active = r.d < a.dim && r.l0 < r.l1;
  return r;
}

// ----------------------------------------------------------------- backward
// Step k holds positions [lk, lk + C).  g of step k is computed when it arrives; dx of
// step k-1 is then complete (it needs g up to W-1 positions later) and is stored.  After
// the last step of the segment, the W-1 positions past it (when inside the sequence)
// are streamed in as one more step to finish dx of the last step.
template <typename T, int W, bool SILU, bool SEQ, int P, int NT>
__global__ void __launch_bounds__(NT) bwd_rows_kernel(const ConvArgs a) {
  constexpr int C = RowStep<T>::C;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowStep<T>* xring = reinterpret_cast<RowStep<T>*>(smem_raw) + threadIdx.x;
  RowStep<T>* gring = reinterpret_cast<RowStep<T>*>(smem_raw) + P * NT + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (unit >= a.units) return;  // whole warps
  const RowLane rl = row_lane<C>(a, unit, lane);
  const int64_t b = rl.b, d = rl.d, l0 = rl.l0, l1 = rl.l1, L = a.seqlen;
  const int64_t tail0 = L - (W - 1);
  float dw[W], db = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) dw[w] = 0.f;

  if (rl.active) {
    const T* xrow = static_cast<const T*>(a.x.data) + b * a.x.s0 + d * a.x.s1;
    const T* grow = static_cast<const T*>(a.dout.data) + b * a.dout.s0 + d * a.dout.s1;
    T* dxrow = static_cast<T*>(a.dx.data) + b * a.dx.s0 + d * a.dx.s1;
    const int nmain = static_cast<int>((l1 - l0 + C - 1) / C);
    const int nall = nmain + (l1 < L ? 1 : 0);  // one more step for the right halo
    auto count_of = [&](int k) {  // positions of step k that carry data
      const int64_t lk = l0 + (int64_t)k * C;
      const int64_t lim = k < nmain ? l1 : min(L, l1 + (W - 1));
      return static_cast<int>(max((int64_t)0, min((int64_t)C, lim - lk)));
    };
    const T* xs_src = xrow + l0;
    const T* gs_src = grow + l0;
#pragma unroll
    for (int k = 0; k < P - 1; ++k) {
      if (k < nall) {
        issue_step<T>(xring + k * NT, xs_src, count_of(k));
        issue_step<T>(gring + k * NT, gs_src, count_of(k));
      }
      cp_async_commit();
      xs_src += C;
      gs_src += C;
    }

    float wv[W], bias;
    {
      float wt[W][1], bt[1];
      load_params<W, 1>(a, d, wt, bt);
#pragma unroll
      for (int w = 0; w < W; ++w) wv[w] = wt[w][0];
      bias = bt[0];
    }
    const int* srow = SEQ ? static_cast<const int*>(a.seq_idx.data) + b * a.seq_idx.s0 : nullptr;
    float xw[W - 1];
    int sw[W - 1];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
      const int64_t l = l0 - (W - 1) + k;
      float v = 0.f;
      if (l >= 0) v = to_f32(xrow[l]);
      else if (a.init.data) v = load_any(a.init.data, a.init.dtype, b * a.init.s0 + d * a.init.s1 + (W - 1 + l) * a.init.s2);
      xw[k] = v;
      sw[k] = (SEQ && l >= 0) ? srow[l * a.seq_idx.s1] : -1;
    }
    float gprev[C];  // g of the previous step
    int sprev[C];
#pragma unroll
    for (int i = 0; i < C; ++i) {
      gprev[i] = 0.f;
      sprev[i] = -1;
    }
    const bool want_dinit = l0 == 0 && a.dinit.data != nullptr;

    for (int k = 0; k < nall; ++k) {
      const int64_t lk = l0 + (int64_t)k * C;
      const int kp = k + P - 1;
      if (kp < nall) {
        issue_step<T>(xring + (kp % P) * NT, xs_src, count_of(kp));
        issue_step<T>(gring + (kp % P) * NT, gs_src, count_of(kp));
      }
      xs_src += C;
      gs_src += C;
      cp_async_commit();
      cp_async_wait<P - 1>();
      const int count = count_of(k);
      float xs[W - 1 + C], gcur[C];
      int ss[W - 1 + C];
#pragma unroll
      for (int q = 0; q < W - 1; ++q) {
        xs[q] = xw[q];
        ss[q] = sw[q];
      }
      {
        float f[C];
        step_to_f32<T>(xring[(k % P) * NT], f);
#pragma unroll
        for (int i = 0; i < C; ++i) xs[W - 1 + i] = f[i];
        step_to_f32<T>(gring[(k % P) * NT], gcur);
      }
#pragma unroll
      for (int i = 0; i < C; ++i) {
        if constexpr (SEQ) ss[W - 1 + i] = i < count ? srow[(lk + i) * a.seq_idx.s1] : -1;
        else ss[W - 1 + i] = 0;
      }
      // g at this step's positions (zero where no data: past L, or past the halo)
#pragma unroll
      for (int i = 0; i < C; ++i) {
        float gv = gcur[i];
        if constexpr (SILU) {
          float p = bias;
#pragma unroll
          for (int w = 0; w < W; ++w) {
            float xin = xs[i + w];
            if constexpr (SEQ) xin = (ss[i + w] == ss[W - 1 + i]) ? xin : 0.f;
            p = fmaf(wv[w], xin, p);
          }
          if constexpr (SEQ) p = (ss[W - 1 + i] >= 0) ? p : 0.f;
          gv *= silu_grad(p);
        }
        if constexpr (SEQ) gv = (ss[W - 1 + i] >= 0) ? gv : 0.f;
        gcur[i] = gv;
      }
      if (k < nmain) {  // dweight / dbias terms of this segment's positions
#pragma unroll
        for (int i = 0; i < C; ++i) {
          db += gcur[i];
#pragma unroll
          for (int w = 0; w < W; ++w) {
            float xin = xs[i + w];
            if constexpr (SEQ) xin = (ss[i + w] == ss[W - 1 + i]) ? xin : 0.f;
            dw[w] = fmaf(gcur[i], xin, dw[w]);
          }
        }
      }
      // dx of the previous step (positions lk - C .. lk - 1): needs g up to W-1 later
      if (k > 0 || want_dinit) {
        float gx[C + W - 1];
        int sx[C + W - 1];
#pragma unroll
        for (int i = 0; i < C; ++i) {
          gx[i] = gprev[i];
          sx[i] = sprev[i];
        }
#pragma unroll
        for (int q = 0; q < W - 1; ++q) {
          gx[C + q] = gcur[q];
          sx[C + q] = ss[W - 1 + q];
        }
        float dxv[C];
#pragma unroll
        for (int i = 0; i < C; ++i) {
          float s = 0.f;
#pragma unroll
          for (int q = 0; q < W; ++q) {
            float gq = gx[i + q];
            if constexpr (SEQ) gq = (sx[i] == sx[i + q]) ? gq : 0.f;
            s = fmaf(wv[W - 1 - q], gq, s);
          }
          dxv[i] = s;
        }
        const int64_t e0 = lk - C;
        if (k > 0) {
          if (a.dfinal.data && e0 + C > tail0) {
#pragma unroll
            for (int i = 0; i < C; ++i)
              if (e0 + i >= tail0 && e0 + i < L)
                dxv[i] += load_any(a.dfinal.data, a.dfinal.dtype, b * a.dfinal.s0 + d * a.dfinal.s1 + (e0 + i - tail0) * a.dfinal.s2);
          }
          store_step<T>(dxrow + e0, f32_to_step<T>(dxv), static_cast<int>(min((int64_t)C, (int64_t)l1 - e0)));
        } else {
          // first step of the first segment: the W-1 positions before 0 -> dinitial
#pragma unroll
          for (int q = 0; q < W - 1; ++q) {
            const int64_t e = q - (W - 1);
            float s = dxv[C - (W - 1) + q];
            if constexpr (SEQ) s = 0.f;
            if (a.dfinal.data && e >= tail0)
              s += load_any(a.dfinal.data, a.dfinal.dtype, b * a.dfinal.s0 + d * a.dfinal.s1 + (e - tail0) * a.dfinal.s2);
            store_any(a.dinit.data, a.dinit.dtype, b * a.dinit.s0 + d * a.dinit.s1 + q * a.dinit.s2, s);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < C; ++i) {
        gprev[i] = gcur[i];
        sprev[i] = ss[W - 1 + i];
      }
#pragma unroll
      for (int q = 0; q < W - 1; ++q) {
        xw[q] = xs[C + q];
        sw[q] = ss[C + q];
      }
    }
    // the segment ends at L: dx of the last step has no positions after it
    if (l1 == L) {
      const int64_t e0 = l0 + (int64_t)(nall - 1) * C;
      float dxv[C];
#pragma unroll
      for (int i = 0; i < C; ++i) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < W; ++q) {
          const float gq = (i + q < C) ? gprev[i + q] : 0.f;
          float gm = gq;
          if constexpr (SEQ) gm = (i + q < C && sprev[i] == sprev[i + q]) ? gq : 0.f;
          s = fmaf(wv[W - 1 - q], gm, s);
        }
        if (a.dfinal.data && e0 + i >= tail0 && e0 + i < L)
          s += load_any(a.dfinal.data, a.dfinal.dtype, b * a.dfinal.s0 + d * a.dfinal.s1 + (e0 + i - tail0) * a.dfinal.s2);
        dxv[i] = s;
      }
      store_step<T>(dxrow + e0, f32_to_step<T>(dxv), static_cast<int>(min((int64_t)C, (int64_t)L - e0)));
    }
  }
  cp_async_wait<0>();

  // dweight / dbias partial sums of this warp unit (summed by reduce_unit_partials)
  // (slab of the unit: value-major, [W + 1][32 lanes], so every store is one 128-byte line)
  float* mine = a.partials + unit * 32 * (W + 1) + lane;
#pragma unroll
  for (int w = 0; w < W; ++w) mine[w * 32] = dw[w];
  mine[W * 32] = db;
}

// ----------------------------------------------------------------- dispatch
template <typename T, int W>
static cudaError_t launch_rows_w(const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  const bool silu = ls.silu, seq = ls.seq;
  {
#define CC1D_GO(SI, SQ) bwd_rows_kernel<T, W, SI, SQ, kRowDepthBwd, kStreamThreads><<<ls.grid, kStreamThreads, ls.smem, s>>>(a)
    if (silu) { if (seq) CC1D_GO(true, true); else CC1D_GO(true, false); }
    else { if (seq) CC1D_GO(false, true); else CC1D_GO(false, false); }
#undef CC1D_GO
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return CC1D_DT_NAME(reduce_rows)(a, W, s);
  }
}

// Backward of (batch, dim, seqlen)-contiguous tensors (the forward uses fwd_row_kernel).
cudaError_t CC1D_DT_NAME(rows)(bool bwd, const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  if (!bwd) return cudaErrorInvalidValue;
  switch (ls.width) {
    case 2: return launch_rows_w<CC1D_DT_TYPE, 2>(a, ls, s);
    case 3: return launch_rows_w<CC1D_DT_TYPE, 3>(a, ls, s);
    case 4: return launch_rows_w<CC1D_DT_TYPE, 4>(a, ls, s);
    default: return cudaErrorInvalidValue;
  }
}

const void* CC1D_DT_NAME(rows_kernel_ptr)(bool bwd) {
  (void)bwd;
  return reinterpret_cast<const void*>(bwd_rows_kernel<CC1D_DT_TYPE, 4, true, false, kRowDepthBwd, kStreamThreads>);
}

}  // namespace cc1d
