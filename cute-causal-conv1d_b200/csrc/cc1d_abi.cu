// extern "C" launchers of libcc1d_b200.so: argument validation, kernel selection,
// launch geometry.  See include/causal_conv1d_b200.h for the contract.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "cc1d_launch.h"
#include "cc1d_update_launch.h"

namespace cc1d {
namespace {

thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};

cc1d_status fail(cc1d_status code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
cc1d_status fail(cc1d_status code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

cc1d_status cuda_fail(cudaError_t e, const char* what) {
  return fail(CC1D_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool is_float(int dt) { return dt == CC1D_FLOAT32 || dt == CC1D_FLOAT16 || dt == CC1D_BFLOAT16; }
int elem_size(int dt) { return dt == CC1D_FLOAT32 ? 4 : (dt == CC1D_INT64 ? 8 : (dt == CC1D_INT32 ? 4 : 2)); }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int pow2_ceil(int64_t v) {
  int p = 1;
  while (p < v && p < (1 << 30)) p <<= 1;
  return p;
}
int log2i(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}

// Stride s of a dimension of extent n keeps vec-element packets aligned (an extent-1
// dimension never moves the pointer, whatever its stride).
bool stride_ok(int64_t s, int64_t n, int vec) { return n <= 1 || s % vec == 0; }

// 16-byte packets along dim (channel-last) are legal for this (B, D, L) tensor.
bool packet_ok_channel_last(const cc1d_tensor& t, int64_t B, int64_t dim, int64_t L) {
  const int vec = 16 / elem_size(t.dtype);
  return t.stride[1] == 1 && dim % vec == 0 && aligned16(t.data) && stride_ok(t.stride[0], B, vec) &&
         stride_ok(t.stride[2], L, vec);
}
// 16-byte packets along seqlen (rows) are legal for this (B, D, L) tensor.
bool packet_ok_rows(const cc1d_tensor& t, int64_t B, int64_t D) {
  const int vec = 16 / elem_size(t.dtype);
  return t.stride[2] == 1 && aligned16(t.data) && stride_ok(t.stride[0], B, vec) && stride_ok(t.stride[1], D, vec);
}

// Packets of `bytes` along dim (channel-last) are legal for this (B, D, L) tensor.
// The streamed kernels index warp units, columns and positions in 32 bits.
constexpr int64_t kMax32 = (int64_t{1} << 31) - 1;

bool stream_ok(const cc1d_tensor& t, int64_t B, int64_t dim, int64_t L, int bytes) {
  const int vec = bytes / elem_size(t.dtype);
  return t.stride[1] == 1 && dim % vec == 0 && (reinterpret_cast<uintptr_t>(t.data) % bytes) == 0 &&
         stride_ok(t.stride[0], B, vec) && stride_ok(t.stride[2], L, vec) && L <= kMax32 && B * dim <= kMax32;
}

// (batch, dim, seqlen)-contiguous rows whose starts are 16-byte aligned.
bool rows_stream_ok(const cc1d_tensor& t, int64_t B, int64_t D, int64_t L) {
  const int vec = 16 / elem_size(t.dtype);
  return t.stride[2] == 1 && aligned16(t.data) && stride_ok(t.stride[0], B, vec) && stride_ok(t.stride[1], D, vec) &&
         L <= kMax32 && B * D <= kMax32;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Resident CTAs per SM for a kernel (cached per device and kernel).
int blocks_per_sm(const void* kernel, size_t smem, int threads = kThreads) {
  static std::mutex mu;
  static struct Entry { int dev; const void* k; size_t smem; int blocks; } entries[256];
  static int n_entries = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_entries; ++i)
    if (entries[i].dev == dev && entries[i].k == kernel && entries[i].smem == smem) return entries[i].blocks;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, smem) != cudaSuccess || blocks < 1) {
    cudaGetLastError();
    blocks = 1;
  }
  if (n_entries < 256) entries[n_entries++] = Entry{dev, kernel, smem, blocks};
  return blocks;
}

const void* kernel_ptr(bool bwd, int dtype, const LaunchShape& ls) {
  if (ls.layout == kLayoutRowWalk) {
    switch (dtype) {
      case CC1D_FLOAT32: return rowwalk_kernel_ptr_f32(bwd, ls.smem);
      case CC1D_FLOAT16: return rowwalk_kernel_ptr_f16(bwd, ls.smem);
      default: return rowwalk_kernel_ptr_bf16(bwd, ls.smem);
    }
  }
  if (ls.layout == kLayoutRowStream) {
    switch (dtype) {
      case CC1D_FLOAT32: return rows_kernel_ptr_f32(bwd);
      case CC1D_FLOAT16: return rows_kernel_ptr_f16(bwd);
      default: return rows_kernel_ptr_bf16(bwd);
    }
  }
  switch (dtype) {
    case CC1D_FLOAT32: return bwd ? bwd_kernel_ptr_f32(ls) : fwd_kernel_ptr_f32(ls);
    case CC1D_FLOAT16: return bwd ? bwd_kernel_ptr_f16(ls) : fwd_kernel_ptr_f16(ls);
    default: return bwd ? bwd_kernel_ptr_bf16(ls) : fwd_kernel_ptr_bf16(ls);
  }
}

cudaError_t dispatch(bool bwd, int dtype, const ConvArgs& a, const LaunchShape& ls, cudaStream_t s) {
  if (ls.layout == kLayoutRowWalk) {
    switch (dtype) {
      case CC1D_FLOAT32: return rowwalk_f32(bwd, a, ls, s);
      case CC1D_FLOAT16: return rowwalk_f16(bwd, a, ls, s);
      default: return rowwalk_bf16(bwd, a, ls, s);
    }
  }
  if (ls.layout == kLayoutRowStream) {
    switch (dtype) {
      case CC1D_FLOAT32: return rows_f32(bwd, a, ls, s);
      case CC1D_FLOAT16: return rows_f16(bwd, a, ls, s);
      default: return rows_bf16(bwd, a, ls, s);
    }
  }
  switch (dtype) {
    case CC1D_FLOAT32: return bwd ? bwd_f32(a, ls, s) : fwd_f32(a, ls, s);
    case CC1D_FLOAT16: return bwd ? bwd_f16(a, ls, s) : fwd_f16(a, ls, s);
    default: return bwd ? bwd_bf16(a, ls, s) : fwd_bf16(a, ls, s);
  }
}

// Launch geometry shared by the forward and backward conv kernels.  It depends only on
// the problem (not on the device) except for the final grid size.
struct Geometry {
  LaunchShape ls;
  ConvArgs a;             // geometry fields only
  int64_t ntiles;
  int64_t nslots;         // backward partial slots per channel tile
  int64_t ncounters;      // backward channel tiles (arrival counters)
  int64_t partial_floats; // backward workspace floats for partial sums
};

Geometry plan(bool bwd, int64_t B, int64_t D, int64_t L, int width, int layout, bool packet, int es) {
  Geometry g;
  std::memset(&g, 0, sizeof(g));
  g.ls.width = width;
  g.ls.layout = layout;
  g.ls.packet = packet;
  const int vec = packet ? 16 / es : 1;
  if (layout == kLayoutChannelLast) {
    const int64_t nv = (D + vec - 1) / vec;
    const int TX = (int)std::min<int64_t>(32, pow2_ceil(nv));
    const int TY = kThreads / TX;
    int64_t chunk = 64;
    if (bwd) {
      // keep the partial slots (batch x sequence tiles) moderate
      while (B * ((((L + chunk - 1) / chunk) + TY - 1) / TY) > 64 && chunk < (1 << 20)) chunk *= 2;
    }
    g.a.tx_shift = log2i(TX);
    g.a.nv = nv;
    g.a.chunk = chunk;
    g.a.nbx = (nv + TX - 1) / TX;
    g.a.nby = (((L + chunk - 1) / chunk) + TY - 1) / TY;
    g.ntiles = g.a.nbx * g.a.nby * B;
    g.nslots = g.a.nby * B;
    g.ncounters = g.a.nbx;
    g.partial_floats = g.nslots * D * (width + 1);
    g.ls.smem = bwd ? (size_t)kThreads * vec * (width + 1) * sizeof(float) : 0;
  } else {
    const int gmin = vec == 1 ? 4 : 1;  // a round must span at least W-1 positions
    const int G = (int)std::max<int64_t>(gmin, std::min<int64_t>(32, pow2_ceil((L + vec - 1) / vec)));
    const int DPB = kThreads / G;
    const int64_t span = (int64_t)G * vec;
    const int64_t rounds_per_row = (L + span - 1) / span;
    int64_t rounds = std::min<int64_t>(rounds_per_row, 8);
    if (rounds < 1) rounds = 1;
    int64_t nck = (rounds_per_row + rounds - 1) / rounds;
    if (nck < 1) nck = 1;
    g.a.g_shift = log2i(G);
    g.a.rounds = (int)rounds;
    g.a.chunk = rounds * span;
    g.a.nck = nck;
    g.a.nbx = (D + DPB - 1) / DPB;
    g.ntiles = g.a.nbx * nck * B;
    g.nslots = nck * B;
    g.ncounters = g.a.nbx;
    g.partial_floats = g.nslots * D * (width + 1);
    g.ls.smem = 0;
  }
  return g;
}

// Number of warp units for `ncol` columns of `len` steps each (at most max_seg segments
// per column) on `target` resident warps.  Estimated time ~ waves x (longest segment +
// per-unit start-up cost, in steps); among one-wave and multi-wave splits pick the
// smallest estimate (ties: fewer units).
int64_t choose_units(int64_t ncol, int64_t len, int64_t max_seg, int64_t target, int64_t unit_overhead,
                     int64_t max_waves) {
  auto cost = [&](int64_t u) {
    const int64_t q = u / ncol;  // every column has at least q segments
    return ((u + target - 1) / target) * ((len + q - 1) / q + unit_overhead);
  };
  int64_t units = std::min<int64_t>(std::max<int64_t>(target, ncol), ncol * max_seg);
  int64_t best = cost(units);
  for (int64_t k = 1; k <= max_waves; ++k) {
    const int64_t cands[2] = {k * target, ((k * target) / ncol) * ncol};
    for (int64_t u : cands) {
      if (u < ncol || u > ncol * max_seg) continue;
      const int64_t c = cost(u);
      if (c < best || (c == best && u < units)) {
        best = c;
        units = u;
      }
    }
  }
  return units;
}

#ifndef CC1D_MIN_ROWS_FWD
#define CC1D_MIN_ROWS_FWD 16
#endif
#ifndef CC1D_MIN_ROWS_BWD
#define CC1D_MIN_ROWS_BWD 32
#endif
#ifndef CC1D_SPREAD_UNITS
#define CC1D_SPREAD_UNITS 1
#endif
// Streamed channel-last kernels: one wave of warps.  A warp column (32 packets of one
// batch row) is cut into seg_q or seg_q+1 sequence segments so that the number of warp
// units equals the resident warp capacity and every warp gets the same number of rows
// (+-1 row, +-1 segment length between columns).
Geometry plan_stream(bool bwd, int64_t B, int64_t D, int64_t L, int width, int es, int64_t resident_blocks,
                     bool small = false, bool many_waves = false) {
  Geometry g;
  std::memset(&g, 0, sizeof(g));
  g.ls.width = width;
  g.ls.layout = kLayoutStream;
  g.ls.packet = true;
  g.ls.small = small;
  const int vec = (bwd ? kBwdPacketBytes : kFwdPacketBytes) / es;  // bytes of channels per lane and row
  const int64_t nv = D / vec;
  const int64_t warps_per_block = (bwd ? kBwdStreamThreads : small ? kFwdStreamThreadsSmall : kFwdStreamThreads) / 32;
  const int64_t ncol = B * ((nv + 31) / 32);
  const int64_t min_rows = bwd ? CC1D_MIN_ROWS_BWD : CC1D_MIN_ROWS_FWD;  // shortest segment
  const int64_t max_seg = std::max<int64_t>(1, L / min_rows);
  const int64_t target = std::max<int64_t>(1, resident_blocks * warps_per_block);
  // Several waves of units let the SMs that draw more DRAM service take more of them.
  // Up to 4 waves, each unit costed 24 rows of start-up; the plain forward goes up to 16
  // waves at 2 rows (config 5 forward: 694 instead of 710-715 us; the backward measured
  // slower with more waves: 1023 -> 1090 us at 16).
  const int64_t units = many_waves ? choose_units(ncol, L, max_seg, target, /*unit_overhead=*/2, /*max_waves=*/16)
                                   : choose_units(ncol, L, max_seg, target, /*unit_overhead=*/24, /*max_waves=*/4);
  g.a.nv = nv;
  g.a.ncol = ncol;
  g.a.seg_q = units / ncol;
  g.a.seg_r = units % ncol;
  g.a.units = units;
  // CTAs: enough for every unit, and at least one per SM when there are that many units
  // (the kernels hand units to warps round robin over the CTAs)
  g.ntiles = (units + warps_per_block - 1) / warps_per_block;
  if (CC1D_SPREAD_UNITS) g.ntiles = std::max<int64_t>(g.ntiles, std::min<int64_t>(units, resident_blocks));
  g.ncounters = 0;  // partials are summed by a second kernel
  g.partial_floats = units * 32 * vec * (width + 1);
  g.ls.smem = bwd     ? (size_t)kStreamDepth * kBwdStreamThreads * 2 * kBwdPacketBytes  // x and dout rings
              : small ? (size_t)kStreamDepthFwdSmall * kFwdStreamThreadsSmall * kFwdPacketBytes
                      : (size_t)kStreamDepthFwd * kFwdStreamThreads * kFwdPacketBytes;
  return g;
}

// Row-stream kernels ((B, D, L) contiguous): lane = channel, warp = 32 channels of one
// batch row and a segment of 32-byte steps along the sequence.
Geometry plan_rows(bool bwd, int64_t B, int64_t D, int64_t L, int width, int es, int64_t resident_blocks) {
  Geometry g;
  std::memset(&g, 0, sizeof(g));
  g.ls.width = width;
  g.ls.layout = kLayoutRowStream;
  g.ls.packet = true;
  const int64_t C = 32 / es;
  const int64_t ncol = B * ((D + 31) / 32);
  const int64_t nsteps = (L + C - 1) / C;
  const int64_t max_seg = std::max<int64_t>(1, nsteps / (bwd ? 4 : 2));
  const int64_t target = std::max<int64_t>(1, resident_blocks * (kStreamThreads / 32));
  const int64_t units = choose_units(ncol, nsteps, max_seg, target, /*unit_overhead=*/4, /*max_waves=*/4);
  g.a.nv = D;  // one channel per lane
  g.a.ncol = ncol;
  g.a.seg_q = units / ncol;
  g.a.seg_r = units % ncol;
  g.a.units = units;
  g.ntiles = (units + kStreamThreads / 32 - 1) / (kStreamThreads / 32);
  g.ncounters = 0;  // partials are summed by a second kernel
  g.partial_floats = units * 32 * (width + 1);
  g.ls.smem = (size_t)2 * kRowDepthBwd * kStreamThreads * 32;
  return g;
}

// Row walk ((B, D, L) contiguous, lanes along the sequence): waves of warps, each
// walking an equal share of the rows x steps sequence (see cc1d_rowwalk.cu).
Geometry plan_rowwalk(bool bwd, int64_t B, int64_t D, int64_t L, int width, int es, int64_t resident_blocks) {
  Geometry g;
  std::memset(&g, 0, sizeof(g));
  g.ls.width = width;
  g.ls.layout = kLayoutRowWalk;
  g.ls.packet = true;
  const int64_t vec = 16 / es;
  const int64_t steps = (L + 32 * vec - 1) / (32 * vec);
  const int64_t total = B * D * steps;
  const int64_t warps_per_block = kRowWalkThreads / 32;
  // The forward walks in several waves of warps when each warp keeps at least ~96 steps
  // (up to 16): SMs that draw more DRAM service then take more warps.  Config 5 contiguous
  // forward: 758 -> 685 us (bf16 W=4), 744 -> 669 us (fp16 W=2); (4, 4096, 8192) takes 2
  // waves (102 -> 98 us; 16 waves there: 129 us).  The backward measured mixed and keeps one.
  const int64_t resident_warps = resident_blocks * warps_per_block;
  const int64_t waves = bwd ? 1 : std::max<int64_t>(1, std::min<int64_t>(16, total / (resident_warps * 96)));
  const int64_t nw = std::max<int64_t>(1, std::min<int64_t>(waves * resident_warps, total));
  g.a.nck = steps;
  g.a.units = total;
  g.a.ncol = nw;
  g.ntiles = (nw + warps_per_block - 1) / warps_per_block;
  g.ncounters = 0;  // partials are summed by a second kernel
  g.partial_floats = bwd ? (D + nw) * (width + 1) : 0;
  g.ls.smem = (size_t)(bwd ? 2 : 1) * kRowWalkDepth * kRowWalkThreads * 16;
  return g;
}

// (batch, dim, seqlen)-contiguous rows for the row walk: 16-byte aligned base and
// strides, seqlen a whole number of packets, 32-bit step counts.
bool rowwalk_ok(const cc1d_tensor& t, int64_t B, int64_t D, int64_t L) {
  const int vec = 16 / elem_size(t.dtype);
  const int64_t steps = (L + 32 * vec - 1) / (32 * vec);
  return t.stride[2] == 1 && aligned16(t.data) && stride_ok(t.stride[0], B, vec) && stride_ok(t.stride[1], D, vec) &&
         L % vec == 0 && B * D * steps <= kMax32;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int64_t bwd_workspace_for(const Geometry& g) {
  const int64_t part = round_up(g.partial_floats * (int64_t)sizeof(float), 256);
  return part + round_up(g.ncounters * (int64_t)sizeof(unsigned int), 256);
}

cc1d_status check_conv_common(int64_t B, int64_t D, int64_t L, int64_t W, const cc1d_tensor& x,
                              const cc1d_tensor& weight, const cc1d_tensor& bias, const cc1d_tensor& seq,
                              const cc1d_tensor& init) {
  if (B < 0 || D < 0 || L < 0) return fail(CC1D_ERR_VALUE, "batch, dim and seqlen must be >= 0");
  if (W < 2 || W > 4) return fail(CC1D_ERR_VALUE, "width must be 2, 3, or 4 (got %lld)", (long long)W);
  if (!is_float(x.dtype)) return fail(CC1D_ERR_TYPE, "x must be float32, float16, or bfloat16");
  if (!is_float(weight.dtype)) return fail(CC1D_ERR_TYPE, "weight must be float32, float16, or bfloat16");
  if (bias.data && !is_float(bias.dtype)) return fail(CC1D_ERR_TYPE, "bias must be a float tensor");
  if (seq.data && seq.dtype != CC1D_INT32) return fail(CC1D_ERR_TYPE, "seq_idx must be int32");
  if (init.data && !is_float(init.dtype)) return fail(CC1D_ERR_TYPE, "initial_states must be a float tensor");
  if (B * D * L > 0 && (!x.data || !weight.data)) return fail(CC1D_ERR_VALUE, "x and weight are required");
  return CC1D_OK;
}

}  // namespace

void set_last_error(const char* msg) { g_last_error = msg; }

cudaError_t allow_dynamic_smem(const void* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static struct Entry { const void* k; int dev; size_t bytes; } done[256];
  static int n = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (done[i].k == kernel && done[i].dev == dev && done[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return e;
  if (n < 256) done[n++] = Entry{kernel, dev, bytes};
  return cudaSuccess;
}

}  // namespace cc1d

using namespace cc1d;

extern "C" {

const char* cc1d_last_error(void) { return g_last_error.c_str(); }

const char* cc1d_status_string(int status) {
  switch (status) {
    case CC1D_OK: return "CC1D_OK";
    case CC1D_ERR_VALUE: return "CC1D_ERR_VALUE";
    case CC1D_ERR_TYPE: return "CC1D_ERR_TYPE";
    case CC1D_ERR_NOT_IMPLEMENTED: return "CC1D_ERR_NOT_IMPLEMENTED";
    case CC1D_ERR_CUDA: return "CC1D_ERR_CUDA";
    default: return "CC1D_ERR_UNKNOWN";
  }
}

int cc1d_abi_version(void) { return CC1D_ABI_VERSION; }

int64_t cc1d_launch_count(void) { return g_launches.load(); }

// Validates a forward and plans its launch.  *empty is set when there is nothing to
// launch (no rows, no channels, or seqlen 0 without final states).
static cc1d_status fwd_prepare(const cc1d_fwd_params* p, Geometry* out_g, bool* empty, bool allow_small = true) {
  *empty = true;
  cc1d_status st = check_conv_common(p->batch, p->dim, p->seqlen, p->width, p->x, p->weight, p->bias,
                                     p->seq_idx, p->initial_states);
  if (st != CC1D_OK) return st;
  if (p->out.dtype != p->x.dtype) return fail(CC1D_ERR_TYPE, "out must have x's dtype");
  if (p->final_states.data && !is_float(p->final_states.dtype))
    return fail(CC1D_ERR_TYPE, "final_states must be a float tensor");
  const int64_t B = p->batch, D = p->dim, L = p->seqlen;
  const int W = (int)p->width;
  if (B == 0 || D == 0) return CC1D_OK;
  if (L == 0) {
    if (p->final_states.data) return fail(CC1D_ERR_VALUE, "seqlen must be > 0 when final_states are requested");
    return CC1D_OK;
  }
  if (!p->out.data) return fail(CC1D_ERR_VALUE, "out is required");
  *empty = false;

  int layout = kLayoutChannelLast;
  bool packet = false;
  const int es = elem_size(p->x.dtype);
  Geometry& g = *out_g;
  if (stream_ok(p->x, B, D, L, kFwdPacketBytes) && stream_ok(p->out, B, D, L, kFwdPacketBytes)) {
    // One CTA of 16 warps per SM with a 16-slot ring: measured faster than two CTAs per
    // SM with 8-slot rings (config 2 forward 26.5 -> 25.4 us, config 4 233 -> 228 us),
    // since each warp walks twice the rows for the same start-up.
    g = plan_stream(false, B, D, L, W, es, (int64_t)sm_count(), false, /*many_waves=*/!p->seq_idx.data);
    // Small problems, whose warp units of at least the shortest segment cannot fill one
    // 16-warp CTA per SM: 128-thread CTAs with 8-slot rings, several per SM (measured on
    // (1, 2048, 2048) fp16: 4.9 instead of 5.7 us; (1, 1024, 4096): 6.2 instead of 7.1 us;
    // on larger problems the one-CTA-per-SM configuration is faster).
    const int64_t max_seg = std::max<int64_t>(1, L / CC1D_MIN_ROWS_FWD);
    if (allow_small && g.a.ncol * max_seg < (int64_t)sm_count() * (kFwdStreamThreads / 32)) {
      LaunchShape probe{};
      probe.layout = kLayoutStream;
      probe.small = true;
      probe.smem = (size_t)kStreamDepthFwdSmall * kFwdStreamThreadsSmall * kFwdPacketBytes;
      const int64_t resident =
          (int64_t)blocks_per_sm(kernel_ptr(false, p->x.dtype, probe), probe.smem, kFwdStreamThreadsSmall) * sm_count();
      g = plan_stream(false, B, D, L, W, es, resident, true);
    }
  } else if (!p->seq_idx.data && rowwalk_ok(p->x, B, D, L) && rowwalk_ok(p->out, B, D, L)) {
    LaunchShape probe{};
    probe.layout = kLayoutRowWalk;
    probe.smem = (size_t)kRowWalkDepth * kRowWalkThreads * 16;
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(false, p->x.dtype, probe), probe.smem, kRowWalkThreads) * sm_count();
    g = plan_rowwalk(false, B, D, L, W, es, resident);
  } else {
    if (p->x.stride[1] == 1 && p->out.stride[1] == 1) {
      packet = packet_ok_channel_last(p->x, B, D, L) && packet_ok_channel_last(p->out, B, D, L);
    } else if (p->x.stride[2] == 1 && p->out.stride[2] == 1) {
      layout = kLayoutRows;
      packet = packet_ok_rows(p->x, B, D) && packet_ok_rows(p->out, B, D);
    }
    g = plan(false, B, D, L, W, layout, packet, es);
  }
  ConvArgs& a = g.a;
  a.batch = B;
  a.dim = D;
  a.seqlen = L;
  a.x = tensor_arg(p->x);
  a.weight = tensor_arg(p->weight);
  a.bias = tensor_arg(p->bias);
  a.seq_idx = tensor_arg(p->seq_idx);
  a.init = tensor_arg(p->initial_states);
  a.final_states = tensor_arg(p->final_states);
  a.out = tensor_arg(p->out);
  g.ls.silu = p->silu != 0;
  g.ls.seq = p->seq_idx.data != nullptr;
  if (g.ls.layout == kLayoutStream || g.ls.layout == kLayoutRowStream || g.ls.layout == kLayoutRowWalk) {
    g.ls.grid = dim3((unsigned)g.ntiles);
  } else {
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(false, p->x.dtype, g.ls), g.ls.smem) * sm_count();
    g.ls.grid = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(g.ntiles, resident)));
  }
  return CC1D_OK;
}

static cc1d_status fwd_run(const cc1d_fwd_params* p, const Geometry& g, void* stream) {
  cudaError_t e = dispatch(false, p->x.dtype, g.a, g.ls, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d forward launch");
  g_launches.fetch_add(1);
  return CC1D_OK;
}

cc1d_status cc1d_fwd_launch(const cc1d_fwd_params* p, void* stream) {
  g_last_error.clear();
  if (!p) return fail(CC1D_ERR_VALUE, "params is NULL");
  Geometry g;
  bool empty = true;
  const cc1d_status st = fwd_prepare(p, &g, &empty);
  if (st != CC1D_OK || empty) return st;
  return fwd_run(p, g, stream);
}

static cc1d_status bwd_prepare(const cc1d_bwd_params* p, Geometry* out_g, bool* empty) {
  if (!p) return fail(CC1D_ERR_VALUE, "params is NULL");
  cc1d_status st = check_conv_common(p->batch, p->dim, p->seqlen, p->width, p->x, p->weight, p->bias,
                                     p->seq_idx, p->initial_states);
  if (st != CC1D_OK) return st;
  if (p->dout.dtype != p->x.dtype || p->dx.dtype != p->x.dtype)
    return fail(CC1D_ERR_TYPE, "dout and dx must have x's dtype");
  if (p->dfinal_states.data && !is_float(p->dfinal_states.dtype))
    return fail(CC1D_ERR_TYPE, "dfinal_states must be a float tensor");
  if (p->dinitial_states.data && !is_float(p->dinitial_states.dtype))
    return fail(CC1D_ERR_TYPE, "dinitial_states must be a float tensor");
  if (p->dinitial_states.data && !p->initial_states.data)
    return fail(CC1D_ERR_VALUE, "dinitial_states requires initial_states");
  if (p->bias.data && !p->dbias) return fail(CC1D_ERR_VALUE, "dbias is required when bias is given");
  const int64_t B = p->batch, D = p->dim, L = p->seqlen;
  *empty = (B == 0 || D == 0 || L == 0);
  if (*empty) return CC1D_OK;
  if (!p->dout.data || !p->dx.data || !p->dweight) return fail(CC1D_ERR_VALUE, "dout, dx and dweight are required");
  int layout = kLayoutChannelLast;
  bool packet = false;
  const int es = elem_size(p->x.dtype);
  if (stream_ok(p->x, B, D, L, kBwdPacketBytes) && stream_ok(p->dout, B, D, L, kBwdPacketBytes) &&
      stream_ok(p->dx, B, D, L, kBwdPacketBytes)) {
    LaunchShape probe{};
    probe.layout = kLayoutStream;
    const size_t smem = (size_t)kStreamDepth * kBwdStreamThreads * 2 * kBwdPacketBytes;
    probe.smem = smem;
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(true, p->x.dtype, probe), smem, kBwdStreamThreads) * sm_count();
    *out_g = plan_stream(true, B, D, L, (int)p->width, es, resident);
    return CC1D_OK;
  }
  if (!p->seq_idx.data && rowwalk_ok(p->x, B, D, L) && rowwalk_ok(p->dout, B, D, L) && rowwalk_ok(p->dx, B, D, L)) {
    LaunchShape probe{};
    probe.layout = kLayoutRowWalk;
    probe.smem = (size_t)2 * kRowWalkDepth * kRowWalkThreads * 16;
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(true, p->x.dtype, probe), probe.smem, kRowWalkThreads) * sm_count();
    *out_g = plan_rowwalk(true, B, D, L, (int)p->width, es, resident);
    return CC1D_OK;
  }
  if (p->x.stride[1] != 1 && rows_stream_ok(p->x, B, D, L) && rows_stream_ok(p->dout, B, D, L) &&
      rows_stream_ok(p->dx, B, D, L)) {
    LaunchShape probe{};
    probe.layout = kLayoutRowStream;
    const size_t smem = (size_t)2 * kRowDepthBwd * kStreamThreads * 32;
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(true, p->x.dtype, probe), smem, kStreamThreads) * sm_count();
    *out_g = plan_rows(true, B, D, L, (int)p->width, es, resident);
    return CC1D_OK;
  }
  if (p->x.stride[1] == 1 && p->dout.stride[1] == 1 && p->dx.stride[1] == 1) {
    packet = packet_ok_channel_last(p->x, B, D, L) && packet_ok_channel_last(p->dout, B, D, L) &&
             packet_ok_channel_last(p->dx, B, D, L);
  } else if (p->x.stride[2] == 1 && p->dout.stride[2] == 1 && p->dx.stride[2] == 1) {
    layout = kLayoutRows;
    packet = packet_ok_rows(p->x, B, D) && packet_ok_rows(p->dout, B, D) && packet_ok_rows(p->dx, B, D);
  }
  *out_g = plan(true, B, D, L, (int)p->width, layout, packet, es);
  return CC1D_OK;
}

int64_t cc1d_bwd_workspace_bytes(const cc1d_bwd_params* p) {
  g_last_error.clear();
  Geometry g;
  bool empty = false;
  if (bwd_prepare(p, &g, &empty) != CC1D_OK) return -1;
  if (empty) return 0;
  return bwd_workspace_for(g);
}

cc1d_status cc1d_bwd_launch(const cc1d_bwd_params* p, void* stream) {
  g_last_error.clear();
  Geometry g;
  bool empty = false;
  cc1d_status st = bwd_prepare(p, &g, &empty);
  if (st != CC1D_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t B = p->batch, D = p->dim, L = p->seqlen;
  const int W = (int)p->width;
  if (empty) {
    // no positions: the parameter gradients are zero
    if (B * D == 0 || !p->dweight) return CC1D_OK;
    cudaError_t e = cudaMemsetAsync(p->dweight, 0, D * W * sizeof(float), s);
    if (e == cudaSuccess && p->dbias) e = cudaMemsetAsync(p->dbias, 0, D * sizeof(float), s);
    if (e == cudaSuccess && p->dinitial_states.data) {
      // only possible with L == 0; dinitial then equals dfinal (not expressible as memset)
      return fail(CC1D_ERR_VALUE, "seqlen must be > 0 when dinitial_states are requested");
    }
    return e == cudaSuccess ? CC1D_OK : cuda_fail(e, "causal_conv1d backward zero fill");
  }
  const int64_t need = bwd_workspace_for(g);
  if (!p->workspace || p->workspace_bytes < need)
    return fail(CC1D_ERR_VALUE, "workspace too small: %lld bytes needed", (long long)need);
  if (!aligned16(p->workspace)) return fail(CC1D_ERR_VALUE, "workspace must be 16-byte aligned");
  ConvArgs& a = g.a;
  a.batch = B;
  a.dim = D;
  a.seqlen = L;
  a.x = tensor_arg(p->x);
  a.weight = tensor_arg(p->weight);
  a.bias = tensor_arg(p->bias);
  a.seq_idx = tensor_arg(p->seq_idx);
  a.init = tensor_arg(p->initial_states);
  a.dout = tensor_arg(p->dout);
  a.dfinal = tensor_arg(p->dfinal_states);
  a.dx = tensor_arg(p->dx);
  a.dinit = tensor_arg(p->dinitial_states);
  a.dweight = p->dweight;
  a.dbias = p->bias.data ? p->dbias : nullptr;
  char* ws = static_cast<char*>(p->workspace);
  a.partials = reinterpret_cast<float*>(ws);
  a.counters = reinterpret_cast<unsigned int*>(ws + round_up(g.partial_floats * (int64_t)sizeof(float), 256));
  g.ls.silu = p->silu != 0;
  g.ls.seq = p->seq_idx.data != nullptr;
  cudaError_t e = cudaSuccess;
  if (g.ncounters > 0) {
    e = cudaMemsetAsync(a.counters, 0, g.ncounters * sizeof(unsigned int), s);
    if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d backward counter reset");
  }
  if (g.ls.layout == kLayoutStream || g.ls.layout == kLayoutRowStream || g.ls.layout == kLayoutRowWalk) {
    g.ls.grid = dim3((unsigned)g.ntiles);
  } else {
    const int64_t resident = (int64_t)blocks_per_sm(kernel_ptr(true, p->x.dtype, g.ls), g.ls.smem) * sm_count();
    g.ls.grid = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(g.ntiles, resident)));
  }
  e = dispatch(true, p->x.dtype, a, g.ls, s);
  if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d backward launch");
  // the streamed layouts add a second kernel that sums the partials
  g_launches.fetch_add(g.ls.layout == kLayoutStream || g.ls.layout == kLayoutRowStream || g.ls.layout == kLayoutRowWalk ? 2 : 1);
  return CC1D_OK;
}

cc1d_status cc1d_update_launch(const cc1d_update_params* p, void* stream) {
  g_last_error.clear();
  if (!p) return fail(CC1D_ERR_VALUE, "params is NULL");
  const int64_t B = p->batch, D = p->dim, T = p->seqlen, S = p->state_len, W = p->width;
  if (B < 0 || D < 0 || T < 0 || S < 0 || p->state_batch < 0) return fail(CC1D_ERR_VALUE, "sizes must be >= 0");
  if (W < 2 || W > 4) return fail(CC1D_ERR_VALUE, "width must be 2, 3, or 4");
  if (S < W - 1) return fail(CC1D_ERR_VALUE, "conv_state is shorter than the convolution history");
  if (B > kMax32 || T > kMax32 || S > kMax32 || p->state_batch > kMax32)
    return fail(CC1D_ERR_VALUE, "update sizes must be below 2^31");
  if (!is_float(p->x.dtype)) return fail(CC1D_ERR_TYPE, "x must be float32, float16, or bfloat16");
  if (!is_float(p->weight.dtype)) return fail(CC1D_ERR_TYPE, "weight must be a float tensor");
  if (p->bias.data && !is_float(p->bias.dtype)) return fail(CC1D_ERR_TYPE, "bias must be a float tensor");
  if (p->conv_state.dtype != p->x.dtype || p->out.dtype != p->x.dtype)
    return fail(CC1D_ERR_TYPE, "conv_state and out must have x's dtype");
  if (p->cache_seqlens.data && p->cache_seqlens.dtype != CC1D_INT32)
    return fail(CC1D_ERR_TYPE, "cache_seqlens must be int32");
  if (p->conv_state_indices.data && p->conv_state_indices.dtype != CC1D_INT32)
    return fail(CC1D_ERR_TYPE, "conv_state_indices must be int32");
  if (!p->conv_state_indices.data && p->state_batch < B)
    return fail(CC1D_ERR_VALUE, "conv_state has fewer rows than the batch");
  if (B == 0 || D == 0 || T == 0) return CC1D_OK;
  if (!p->x.data || !p->conv_state.data || !p->weight.data || !p->out.data)
    return fail(CC1D_ERR_VALUE, "x, conv_state, weight and out are required");
  const bool w_flat16 = p->weight.dtype == CC1D_FLOAT32 && p->weight.stride[1] == 1 && p->weight.stride[0] == W &&
                        aligned16(p->weight.data);
  const bool b_flat16 = p->bias.data && p->bias.dtype == CC1D_FLOAT32 && p->bias.stride[0] == 1 && aligned16(p->bias.data);
  // Single-token decode (seqlen == 1) with channel packets in x/out and a state layout one
  // of the decode kernels takes: every load of a row is issued before any is used.
  if (T == 1 && B * D <= kMax32) {
    const cc1d_tensor& st = p->conv_state;
    const bool circ = p->cache_seqlens.data != nullptr;
    const int es = elem_size(p->x.dtype);
    auto ch_ok = [&](const cc1d_tensor& t, int64_t rows, int ch) {
      return t.stride[1] == 1 && (reinterpret_cast<uintptr_t>(t.data) % (uintptr_t)(ch * es)) == 0 &&
             stride_ok(t.stride[0], rows, ch) && D % ch == 0;
    };
    int kind = -1;
    const int v16 = 16 / es;
    if (ch_ok(p->x, B, v16) && ch_ok(p->out, B, v16)) {
      if (ch_ok(st, p->state_batch, v16) && stride_ok(st.stride[2], S, v16) && (circ || S == W - 1))
        kind = circ ? kDecodeClCirc : kDecodeClShift;
      else if (!circ && S == W - 1 && st.stride[2] == 1 && st.stride[1] == S && aligned16(st.data) &&
               stride_ok(st.stride[0], p->state_batch, v16))
        kind = kDecodeBlock;
    }
    if (kind < 0 && circ && es == 2 && S % 4 == 0 && st.stride[2] == 1 && st.stride[1] == S &&
        (reinterpret_cast<uintptr_t>(st.data) & 7u) == 0 && stride_ok(st.stride[0], p->state_batch, 4)) {
      const int ch = decode_channels_per_thread(kDecodeRing, p->x.dtype);
      if (ch_ok(p->x, B, ch) && ch_ok(p->out, B, ch)) kind = kDecodeRing;
    }
    if (kind >= 0) {
      UpdateArgs a;
      std::memset(&a, 0, sizeof(a));
      a.batch = B;
      a.dim = D;
      a.seqlen = T;
      a.state_len = S;
      a.state_batch = p->state_batch;
      a.x = tensor_arg(p->x);
      a.state = tensor_arg(p->conv_state);
      a.weight = tensor_arg(p->weight);
      a.bias = tensor_arg(p->bias);
      a.out = tensor_arg(p->out);
      a.cache_seqlens = static_cast<const int32_t*>(p->cache_seqlens.data);
      a.cache_stride = p->cache_seqlens.stride[0];
      a.indices = static_cast<const int32_t*>(p->conv_state_indices.data);
      a.indices_stride = p->conv_state_indices.stride[0];
      a.silu = p->silu;
      a.weight_vec = w_flat16;
      a.bias_vec = b_flat16;
      cudaError_t e = launch_decode(p->x.dtype, kind, a, (int)W, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d update launch");
      g_launches.fetch_add(1);
      return CC1D_OK;
    }
  }
  // A shift update (no circular buffer, state_len == W-1) of a state whose entries per
  // channel are contiguous and channels state_len apart: whole 8-byte blocks of
  // channels' histories (update_shift_kernel).
  const int ch = 8 / elem_size(p->x.dtype);
  auto aligned8 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 7u) == 0; };
  auto vec8 = [&](const cc1d_tensor& t, int64_t n0, int64_t n2) {
    return t.stride[1] == 1 && aligned8(t.data) && stride_ok(t.stride[0], n0, ch) && stride_ok(t.stride[2], n2, ch);
  };
  const bool shift = !p->cache_seqlens.data && S == W - 1 && D % ch == 0 && p->conv_state.stride[2] == 1 &&
                     p->conv_state.stride[1] == S && aligned8(p->conv_state.data) &&
                     stride_ok(p->conv_state.stride[0], p->state_batch, ch) && vec8(p->x, B, T) && vec8(p->out, B, T);
  const int vec = 8 / elem_size(p->x.dtype);  // 8-byte packets along dim
  auto ok = [&](const cc1d_tensor& t, int64_t n0, int64_t n2) {
    return t.stride[1] == 1 && (reinterpret_cast<uintptr_t>(t.data) % 8) == 0 && stride_ok(t.stride[0], n0, vec) &&
           stride_ok(t.stride[2], n2, vec);
  };
  const bool packet = D % vec == 0 && ok(p->x, B, T) && ok(p->out, B, T) && ok(p->conv_state, p->state_batch, S);
  UpdateArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = B;
  a.dim = D;
  a.seqlen = T;
  a.state_len = S;
  a.state_batch = p->state_batch;
  a.x = tensor_arg(p->x);
  a.state = tensor_arg(p->conv_state);
  a.weight = tensor_arg(p->weight);
  a.bias = tensor_arg(p->bias);
  a.out = tensor_arg(p->out);
  a.cache_seqlens = static_cast<const int32_t*>(p->cache_seqlens.data);
  a.cache_stride = p->cache_seqlens.stride[0];
  a.indices = static_cast<const int32_t*>(p->conv_state_indices.data);
  a.indices_stride = p->conv_state_indices.stride[0];
  a.silu = p->silu;
  const bool w_flat = p->weight.dtype == CC1D_FLOAT32 && p->weight.stride[1] == 1 && p->weight.stride[0] == W &&
                      aligned16(p->weight.data);
  if (shift) {
    a.weight_vec = w_flat;  // 8-byte weight pairs: d0 * W is even
    const int64_t blocks = ((D / ch + 31) / 32) * ((B + 8 * kUpdateRows - 1) / (8 * kUpdateRows));
    cudaError_t e = launch_update_shift(p->x.dtype, a, (int)W, dim3((unsigned)blocks), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d update launch");
    g_launches.fetch_add(1);
    return CC1D_OK;
  }
  a.weight_vec = packet && (vec * W) % 4 == 0 && w_flat;
  const int64_t nv = (D + (packet ? vec : 1) - 1) / (packet ? vec : 1);
  const int64_t blocks = ((nv + 31) / 32) * ((B + 8 * kUpdateRows - 1) / (8 * kUpdateRows));
  cudaError_t e = launch_update(p->x.dtype, a, (int)W, packet, dim3((unsigned)std::max<int64_t>(1, blocks)),
                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d update launch");
  g_launches.fetch_add(1);
  return CC1D_OK;
}

// Validates a varlen-states gather; *empty is set when there is nothing to write.
static cc1d_status varlen_check(const cc1d_varlen_states_params* p, bool* empty) {
  *empty = true;
  const int64_t B = p->batch, D = p->dim, S = p->state_len;
  if (B < 0 || D < 0 || S < 0 || p->total_tokens < 0) return fail(CC1D_ERR_VALUE, "sizes must be >= 0");
  if (!is_float(p->x.dtype)) return fail(CC1D_ERR_TYPE, "x must be float32, float16, or bfloat16");
  if (p->states.dtype != p->x.dtype) return fail(CC1D_ERR_TYPE, "states must have x's dtype");
  if (p->cu_seqlens.dtype != CC1D_INT32 && p->cu_seqlens.dtype != CC1D_INT64)
    return fail(CC1D_ERR_TYPE, "cu_seqlens must be int32 or int64");
  if (B == 0 || D == 0 || S == 0) return CC1D_OK;
  if (!p->x.data || !p->cu_seqlens.data || !p->states.data)
    return fail(CC1D_ERR_VALUE, "x, cu_seqlens and states are required");
  *empty = false;
  return CC1D_OK;
}

static cc1d_status varlen_run(const cc1d_varlen_states_params* p, void* stream) {
  const int64_t B = p->batch, D = p->dim, S = p->state_len;
  const int vec = 16 / elem_size(p->x.dtype);
  const bool packet = D % vec == 0 && p->x.stride[1] == 1 && p->states.stride[1] == 1 && aligned16(p->x.data) &&
                      aligned16(p->states.data) && stride_ok(p->x.stride[0], p->total_tokens, vec) &&
                      stride_ok(p->states.stride[0], B, vec) && stride_ok(p->states.stride[2], S, vec);
  VarlenArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = B;
  a.dim = D;
  a.state_len = S;
  a.total_tokens = p->total_tokens;
  a.x = tensor_arg(p->x);
  a.states = tensor_arg(p->states);
  a.cu = p->cu_seqlens.data;
  a.cu_stride = p->cu_seqlens.stride[0];
  a.cu_is_64 = p->cu_seqlens.dtype == CC1D_INT64;
  const int64_t items = B * S * ((D + (packet ? vec : 1) - 1) / (packet ? vec : 1));
  const int64_t blocks = std::min<int64_t>((items + kThreads - 1) / kThreads, (int64_t)sm_count() * 8);
  cudaError_t e = launch_varlen_states(p->x.dtype, a, packet, dim3((unsigned)std::max<int64_t>(1, blocks)),
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "causal_conv1d varlen states launch");
  g_launches.fetch_add(1);
  return CC1D_OK;
}

cc1d_status cc1d_varlen_states_launch(const cc1d_varlen_states_params* p, void* stream) {
  g_last_error.clear();
  if (!p) return fail(CC1D_ERR_VALUE, "params is NULL");
  bool empty = true;
  const cc1d_status st = varlen_check(p, &empty);
  if (st != CC1D_OK || empty) return st;
  return varlen_run(p, stream);
}

cc1d_status cc1d_fwd_varlen_states_launch(const cc1d_fwd_varlen_states_params* p, void* stream) {
  g_last_error.clear();
  if (!p) return fail(CC1D_ERR_VALUE, "params is NULL");
  const cc1d_fwd_params& f = p->fwd;
  if (f.batch != 1) return fail(CC1D_ERR_VALUE, "packed sequences need batch == 1 (got %lld)", (long long)f.batch);
  // the gather the forward stands in for: x[0] viewed as (total_tokens = seqlen, dim)
  cc1d_varlen_states_params v;
  std::memset(&v, 0, sizeof(v));
  v.batch = p->nseq;
  v.dim = f.dim;
  v.state_len = p->state_len;
  v.total_tokens = f.seqlen;
  v.x = f.x;
  v.x.stride[0] = f.x.stride[2];
  v.x.stride[1] = f.x.stride[1];
  v.x.stride[2] = 0;
  v.cu_seqlens = p->cu_seqlens;
  v.states = p->states;
  bool no_states = true, no_fwd = true;
  cc1d_status st = varlen_check(&v, &no_states);
  if (st != CC1D_OK) return st;
  Geometry g;
  st = fwd_prepare(&f, &g, &no_fwd, /*allow_small=*/false);  // the state-emitting kernel has one configuration
  if (st != CC1D_OK) return st;
  // The streamed forward writes the states itself when it runs the packed (seq_idx)
  // variant, the sequence positions fit its 32-bit row counters and the states take
  // its packets; otherwise the gather runs as its own launch after the forward.
  const int vec = kFwdPacketBytes / elem_size(f.x.dtype);
  // (seqlen < 2^31 - 1: the kernel clamps offsets to seqlen + 1 in 32-bit arithmetic)
  const bool fused = !no_fwd && !no_states && g.ls.layout == kLayoutStream && f.seq_idx.data &&
                     f.seqlen < kMax32 && p->nseq <= kMax32 && p->state_len <= kMax32 && p->states.stride[1] == 1 &&
                     (reinterpret_cast<uintptr_t>(p->states.data) % kFwdPacketBytes) == 0 &&
                     stride_ok(p->states.stride[0], p->nseq, vec) && stride_ok(p->states.stride[2], p->state_len, vec);
  if (fused) {
    ConvArgs& a = g.a;
    a.states = tensor_arg(p->states);
    a.cu = p->cu_seqlens.data;
    a.cu_stride = p->cu_seqlens.stride[0];
    a.cu_is_64 = p->cu_seqlens.dtype == CC1D_INT64;
    a.nseq = (int)p->nseq;
    a.state_len = (int)p->state_len;
    g.ls.emit = true;
    return fwd_run(&f, g, stream);
  }
  if (!no_fwd && (st = fwd_run(&f, g, stream)) != CC1D_OK) return st;
  if (!no_states) return varlen_run(&v, stream);
  return CC1D_OK;
}

}  // extern "C"
