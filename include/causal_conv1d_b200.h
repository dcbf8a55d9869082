/*
 * causal_conv1d_b200.h -- C ABI of the B200 (sm_100a) causal_conv1d kernels.
 *
 * libcc1d_b200.so exports the launchers below.  They take plain pointers, int64 sizes
 * and int64 element strides, launch asynchronously on the given CUDA stream
 * (a cudaStream_t passed as void*; NULL is the legacy default stream) on the calling
 * thread's current device, never allocate, never synchronise, and return a
 * cc1d_status.  Argument errors are detected on the host before any launch and
 * leave a message for cc1d_last_error().
 *
 * The operator is the depthwise causal convolution
 *     out[b, d, l] = act(bias[d] + sum_{w<W} weight[d, w] * x[b, d, l - (W-1) + w]),
 * W in {2, 3, 4}, act in {identity, SiLU}, fp32 accumulation, with x at negative
 * positions taken from initial_states (or zero).
 *
 * Each entry point cites the reference interface it replaces (paths relative to the
 * root of the reference project, Butterfingrz/cute-causal-conv1d 1.6.2.post1).
 */
#ifndef CAUSAL_CONV1D_B200_H_
#define CAUSAL_CONV1D_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CC1D_ABI_VERSION 1

/* Element types (the dtype field of cc1d_tensor). */
typedef enum cc1d_dtype {
  CC1D_FLOAT32 = 0,
  CC1D_FLOAT16 = 1,
  CC1D_BFLOAT16 = 2,
  CC1D_INT32 = 3,
  CC1D_INT64 = 4
} cc1d_dtype;

/* Return codes.  The Python layer maps them to the exception types the reference
 * raises for the same conditions. */
typedef enum cc1d_status {
  CC1D_OK = 0,
  CC1D_ERR_VALUE = 1,           /* bad shape, size, width or stride   -> ValueError */
  CC1D_ERR_TYPE = 2,            /* unsupported dtype                   -> TypeError */
  CC1D_ERR_NOT_IMPLEMENTED = 3, /* unsupported feature combination     -> NotImplementedError */
  CC1D_ERR_CUDA = 4             /* CUDA runtime error at launch        -> RuntimeError */
} cc1d_status;

/* A strided device tensor of up to three dimensions.  data == NULL means "absent"
 * for optional arguments.  Strides are in elements; unused trailing strides are
 * ignored.  The logical shape of each tensor is fixed by the params struct. */
typedef struct cc1d_tensor {
  void* data;
  int32_t dtype; /* cc1d_dtype */
  int32_t reserved;
  int64_t stride[3];
} cc1d_tensor;

/* ------------------------------------------------------------------- forward
 * Replaces causal_conv1d/cutedsl_kernels.py:336-376 (causal_conv1d_fwd_cutedsl) and
 * the PyTorch fallback causal_conv1d/cpp_functions.py:21-54,64-89
 * (_causal_conv1d_torch + final-state copy); legacy binding
 * csrc/causal_conv1d.cpp:150-258 (causal_conv1d_fwd).
 *
 * Any strides are accepted.  Channel-last x (stride[1] == 1) and (batch, dim, seqlen)
 * contiguous x (stride[2] == 1) get dedicated 128-bit kernels.
 *   x, out          (batch, dim, seqlen)   float32 / float16 / bfloat16, same dtype
 *   weight          (dim, width)           any float dtype
 *   bias            (dim,)                 any float dtype, optional
 *   seq_idx         (batch, seqlen)        int32, optional; tap w of output l is used
 *                                          only if seq_idx[l-(W-1)+w] == seq_idx[l];
 *                                          out = 0 where seq_idx < 0
 *   initial_states  (batch, dim, width-1)  any float dtype, optional (not with seq_idx)
 *   final_states    (batch, dim, width-1)  any float dtype, optional output: the last
 *                                          width-1 entries of [initial_states | x]
 */
typedef struct cc1d_fwd_params {
  int64_t batch, dim, seqlen, width;
  cc1d_tensor x;
  cc1d_tensor weight;
  cc1d_tensor bias;
  cc1d_tensor seq_idx;
  cc1d_tensor initial_states;
  cc1d_tensor final_states;
  cc1d_tensor out;
  int32_t silu;
  int32_t reserved;
} cc1d_fwd_params;

cc1d_status cc1d_fwd_launch(const cc1d_fwd_params* params, void* stream);

/* ------------------------------------------------------------------ backward
 * Replaces causal_conv1d/cutedsl_kernels.py:1618-1649 (causal_conv1d_bwd_cutedsl with
 * its fused/generic kernels and the deterministic reduce, :854-1261) and the autograd
 * fallback causal_conv1d/cpp_functions.py:115-166 (seq_idx, initial_states,
 * dfinal_states); legacy binding csrc/causal_conv1d.cpp:261-463 (causal_conv1d_bwd).
 *
 *   x, weight, bias, seq_idx, initial_states  as in the forward
 *   dout            (batch, dim, seqlen)   x's dtype
 *   dfinal_states   (batch, dim, width-1)  any float dtype, optional
 *   dx              (batch, dim, seqlen)   output, x's dtype, any strides
 *   dinitial_states (batch, dim, width-1)  optional output, any float dtype
 *   dweight         (dim, width) fp32 contiguous output
 *   dbias           (dim,) fp32 output, required iff bias is given
 *   workspace       device scratch of cc1d_bwd_workspace_bytes(params) bytes,
 *                   16-byte aligned, contents need not be initialised
 * dweight/dbias are reduced in a fixed order: results are bit-reproducible for the
 * same inputs and launch configuration, independent of thread scheduling.
 */
typedef struct cc1d_bwd_params {
  int64_t batch, dim, seqlen, width;
  cc1d_tensor x;
  cc1d_tensor weight;
  cc1d_tensor bias;
  cc1d_tensor seq_idx;
  cc1d_tensor initial_states;
  cc1d_tensor dout;
  cc1d_tensor dfinal_states;
  cc1d_tensor dx;
  cc1d_tensor dinitial_states;
  float* dweight;
  float* dbias;
  void* workspace;
  int64_t workspace_bytes;
  int32_t silu;
  int32_t reserved;
} cc1d_bwd_params;

/* Scratch bytes cc1d_bwd_launch needs for these params (0 for empty problems), or
 * -1 with cc1d_last_error() set if the params are invalid. */
int64_t cc1d_bwd_workspace_bytes(const cc1d_bwd_params* params);

cc1d_status cc1d_bwd_launch(const cc1d_bwd_params* params, void* stream);

/* ----------------------------------------- backward without a caller workspace
 * No counterpart in the reference.  For callers that cannot allocate device memory
 * (plugin hosts that pass only the operands, servers with a fixed device-memory budget,
 * code that must not touch the allocator between launches): same contract and results
 * as cc1d_bwd_launch, but params->workspace and params->workspace_bytes are ignored and
 * the scratch comes from a static array of CC1D_STATIC_SCRATCH_BYTES bytes inside the
 * library, so the call allocates nothing.
 *   - Every GPU on which the library is used holds the array until the process exits.
 *   - The first call on a device looks up the array's device address there; make that
 *     first call before capturing a stream.
 *   - All calls share the array: calls that overlap on the GPU race on it.
 *   - A problem needing more scratch than the array holds (cc1d_bwd_workspace_bytes)
 *     is rejected with CC1D_ERR_VALUE before anything is launched.
 */
#define CC1D_STATIC_SCRATCH_BYTES (32 * 1024 * 1024)
/* The device address of the array is looked up once per device and kept for the life of
 * the process: do not use this entry point across a device reset (cudaDeviceReset) in the
 * same process. */

cc1d_status cc1d_bwd_launch_static(const cc1d_bwd_params* params, void* stream);

/* -------------------------------------------------------------------- update
 * Replaces causal_conv1d/cutedsl_kernels.py:554-582 (causal_conv1d_update_cutedsl,
 * kernel :379-493) and the layout fallback causal_conv1d/cpp_functions.py:169-238;
 * legacy binding csrc/causal_conv1d.cpp:466-557 (causal_conv1d_update).
 *
 *   x, out          (batch, dim, seqlen)            same float dtype, any strides
 *   conv_state      (state_batch, dim, state_len)   x's dtype, updated in place
 *   weight, bias    as in the forward
 *   cache_seqlens   (batch,) int32, optional: conv_state is a circular buffer; the
 *                   history is read at (cache_seqlens[b] - (W-1) + i) mod state_len and
 *                   x[t] is written at (cache_seqlens[b] + t) mod state_len
 *   conv_state_indices (batch,) int32, optional: state row of batch row b; a negative
 *                   index gives a zero output row and no state write, and so does an
 *                   index >= state_batch (out of range; the reference leaves it undefined)
 * Without cache_seqlens the state becomes the last state_len entries of [state | x].
 * Requires state_len >= width - 1.
 */
typedef struct cc1d_update_params {
  int64_t batch, dim, seqlen, width, state_batch, state_len;
  cc1d_tensor x;
  cc1d_tensor conv_state;
  cc1d_tensor weight;
  cc1d_tensor bias;
  cc1d_tensor cache_seqlens;
  cc1d_tensor conv_state_indices;
  cc1d_tensor out;
  int32_t silu;
  int32_t reserved;
} cc1d_update_params;

cc1d_status cc1d_update_launch(const cc1d_update_params* params, void* stream);

/* ------------------------------------------------------------- varlen states
 * Replaces causal_conv1d/causal_conv1d_varlen.py:7-11 ->
 * causal_conv1d/cutedsl_kernels.py:660-674 (causal_conv1d_varlen_states_cutedsl,
 * kernel :585-621).
 *
 *   x           (total_tokens, dim)       float dtype, any strides
 *   cu_seqlens  (batch + 1,)              int32 or int64 cumulative sequence offsets
 *   states      (batch, dim, state_len)   output, x's dtype:
 *               states[b, :, s] = x[cu[b+1] - state_len + s] if that row is >= cu[b],
 *               else 0 (bit-exact copy); a row at or past total_tokens gives 0 as well
 *               (cu_seqlens out of range; the reference leaves it undefined).
 */
typedef struct cc1d_varlen_states_params {
  int64_t batch, dim, state_len, total_tokens;
  cc1d_tensor x;
  cc1d_tensor cu_seqlens;
  cc1d_tensor states;
} cc1d_varlen_states_params;

cc1d_status cc1d_varlen_states_launch(const cc1d_varlen_states_params* params, void* stream);

/* ------------------------------------ forward that also writes the varlen states
 * Fuses the two prefill calls of the reference, causal_conv1d_fn over packed sequences
 * (causal_conv1d/causal_conv1d_interface.py:99-129 with seq_idx) followed by
 * causal_conv1d_varlen_states (causal_conv1d/causal_conv1d_varlen.py:7-11), that hand
 * the decode states to causal_conv1d_update.  Same results as
 *     cc1d_fwd_launch(&params->fwd)
 *     cc1d_varlen_states_launch({batch = nseq, dim, state_len, total_tokens = seqlen,
 *                                x = fwd.x[0] as (seqlen, dim), cu_seqlens, states})
 * but with seq_idx given, channel-last x and states whose channel stride is 1, the
 * forward kernel stores each sequence's last state_len rows as it streams them, so x
 * is read once and no second launch is made.  Other arguments take the two launches.
 *   fwd         forward params; fwd.batch must be 1 (sequences packed along seqlen)
 *   nseq        number of sequences
 *   cu_seqlens  (nseq + 1,) int32 or int64, non-decreasing, cu[nseq] <= seqlen (for
 *               other offsets the states of the sequences concerned are unspecified, but
 *               nothing outside the given tensors is read or written)
 *   states      (nseq, dim, state_len) output, x's dtype:
 *               states[k, :, s] = x[0, :, cu[k+1] - state_len + s] if that position is
 *               >= cu[k], else 0 (bit-exact copy)
 */
typedef struct cc1d_fwd_varlen_states_params {
  cc1d_fwd_params fwd;
  int64_t nseq, state_len;
  cc1d_tensor cu_seqlens;
  cc1d_tensor states;
} cc1d_fwd_varlen_states_params;

cc1d_status cc1d_fwd_varlen_states_launch(const cc1d_fwd_varlen_states_params* params, void* stream);

/* ------------------------------------------------------------------- utility */
/* Message of the last error on the calling thread ("" if none). */
const char* cc1d_last_error(void);
/* Static name of a status code. */
const char* cc1d_status_string(int status);
/* CC1D_ABI_VERSION the library was built with. */
int cc1d_abi_version(void);
/* Number of kernel launches made by this process through the launchers above
 * (a diagnostic counter; launches, not completed kernels). */
int64_t cc1d_launch_count(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* CAUSAL_CONV1D_B200_H_ */
