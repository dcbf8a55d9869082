"""Numpy restatement of the reference causal_conv1d algorithm (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may use this
module; it is the parity checker, never the product path.

Arrays use *storage* form: ``float32`` and ``float16`` arrays hold their own values,
``bfloat16`` tensors are ``uint16`` arrays holding the raw bits.  Every function takes
the dtype name of each floating tensor ("float32", "float16", "bfloat16") and returns
outputs in storage form.  Tensors are logical ``(batch, dim, seqlen)`` arrays; memory
layout (channel-last vs contiguous) does not change the arithmetic, so the oracle is
layout-free.

Arithmetic is fp32 throughout, as in the reference's kernels (fp32 accumulation,
``cutedsl_kernels.py:228-239``) and in its oracles when weights are fp32
(``causal_conv1d_interface.py:156``: ``x.to(weight.dtype)``).  Every function cites the
reference code it restates (paths relative to the reference project root).
"""

from __future__ import annotations

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


# ----------------------------------------------------------------------------- dtypes
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bits (uint16) -> float32: the bf16 pattern is the high half of an f32."""
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits with round-to-nearest-even (NaN stays a quiet NaN)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    u = v.view(np.uint32).astype(np.uint64)
    rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    out = rounded.astype(np.uint16)
    nan = np.isnan(v)
    if nan.any():
        out[nan] = ((u[nan] >> np.uint64(16)) | np.uint64(0x40)).astype(np.uint16)
    return out


def to_f32(a: np.ndarray | None, dtype: str) -> np.ndarray | None:
    """Storage array -> float32 values (exact for all three dtypes)."""
    if a is None:
        return None
    if dtype == "bfloat16":
        return bf16_bits_to_f32(np.asarray(a, dtype=np.uint16))
    if dtype in ("float16", "float32"):
        return np.asarray(a).astype(np.float32)
    raise ValueError(f"unsupported dtype {dtype}")


def from_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> storage array of ``dtype`` (round-to-nearest-even)."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "bfloat16":
        return f32_to_bf16_bits(a)
    if dtype == "float16":
        return a.astype(np.float16)
    if dtype == "float32":
        return a.copy()
    raise ValueError(f"unsupported dtype {dtype}")


def _silu(p: np.ndarray) -> np.ndarray:
    # F.silu(p) = p * sigmoid(p)  (causal_conv1d_interface.py:173)
    with np.errstate(over="ignore"):
        return p * (np.float32(1.0) / (np.float32(1.0) + np.exp(-p)))


def _sigmoid(p: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.float32(1.0) / (np.float32(1.0) + np.exp(-p))


# ---------------------------------------------------------------------------- forward
def _tap_masks(seq_idx: np.ndarray | None, width: int, seqlen: int):
    """Per-tap validity masks for packed sequences.

    Restates ``cpp_functions.py:41-51``: tap ``w`` of output ``l`` reads position
    ``l-(W-1)+w`` and is kept only when ``seq_idx`` there equals ``seq_idx[l]`` and
    ``seq_idx[l] >= 0``; positions before the start are padded with -1.
    Returns a list of ``(batch, seqlen)`` bool arrays (or Nones) and the output mask.
    """
    if seq_idx is None:
        return [None] * width, None
    s = np.asarray(seq_idx, dtype=np.int64)
    padded = np.concatenate([np.full((s.shape[0], width - 1), -1, np.int64), s], axis=1)
    cur_ok = s >= 0
    masks = [cur_ok & (padded[:, w : w + seqlen] == s) for w in range(width)]
    return masks, cur_ok


def _extended_input(xf, width, initial_f):
    """``[initial_states | x]`` (or zero left padding), cpp_functions.py:33-36."""
    b, d, _ = xf.shape
    if initial_f is None:
        pre = np.zeros((b, d, width - 1), np.float32)
    else:
        pre = initial_f.astype(np.float32)
    return np.concatenate([pre, xf], axis=2)


def _preact(xe, wf, bf, masks, out_mask, seqlen):
    """Pre-activation ``bias + sum_w w[w] * x[l-(W-1)+w]`` (cpp_functions.py:38-51)."""
    b, d, _ = xe.shape
    width = wf.shape[1]
    acc = np.zeros((b, d, seqlen), np.float32)
    if bf is not None:
        acc = acc + bf[None, :, None]
    for w in range(width):
        term = xe[:, :, w : w + seqlen] * wf[None, :, w, None]
        if masks[w] is not None:
            term = term * masks[w][:, None, :]
        acc = acc + term
    if out_mask is not None:
        acc = acc * out_mask[:, None, :]
    return acc


def final_states_f32(xf, width, initial_f):
    """Last ``W-1`` entries of ``[initial | x]``, left zero padded when shorter.

    Restates ``cpp_functions.py:57-61,82-88`` and ``causal_conv1d_interface.py:165-168``.
    """
    b, d, seqlen = xf.shape
    hist = xf if initial_f is None else np.concatenate([initial_f, xf], axis=2)
    if hist.shape[2] < width - 1:
        pad = np.zeros((b, d, width - 1 - hist.shape[2]), np.float32)
        hist = np.concatenate([pad, hist], axis=2)
    return hist[:, :, hist.shape[2] - (width - 1) :]


def fwd(x, x_dtype, weight, w_dtype, bias=None, b_dtype=None, seq_idx=None,
        initial_states=None, i_dtype=None, silu=False, return_final_states=False,
        final_dtype=None):
    """Forward: ``out = act(bias + sum_w weight[:, w] * x[..., l-(W-1)+w])``.

    Restates ``causal_conv1d_interface.py:135-174`` (``causal_conv1d_ref``) and the
    seq_idx / initial-states path ``cpp_functions.py:21-54,64-89``.
    Returns ``(out, final_states)``; ``final_states`` is None unless requested.
    """
    xf = to_f32(x, x_dtype)
    wf = to_f32(weight, w_dtype)
    bf = to_f32(bias, b_dtype or w_dtype) if bias is not None else None
    init_f = to_f32(initial_states, i_dtype or x_dtype) if initial_states is not None else None
    _, _, seqlen = xf.shape
    width = wf.shape[1]
    masks, out_mask = _tap_masks(seq_idx, width, seqlen)
    xe = _extended_input(xf, width, init_f)
    acc = _preact(xe, wf, bf, masks, out_mask, seqlen)
    if silu:
        acc = _silu(acc)
    out = from_f32(acc, x_dtype)
    final = None
    if return_final_states:
        final = from_f32(final_states_f32(xf, width, init_f), final_dtype or x_dtype)
    return out, final


# --------------------------------------------------------------------------- backward
def bwd(x, x_dtype, weight, w_dtype, dout, bias=None, b_dtype=None, seq_idx=None,
        initial_states=None, i_dtype=None, dfinal_states=None, dfinal_dtype=None,
        silu=False):
    """Backward of :func:`fwd`; returns ``(dx, dweight, dbias, dinitial_states)``.

    Restates autograd through ``_causal_conv1d_torch`` and ``_last_history``
    (``cpp_functions.py:115-166``), which is also what the fused kernels compute
    (``cutedsl_kernels.py:854-1205``):
    ``g = dout * silu'(p)`` (masked by ``seq_idx >= 0``), ``dbias = sum g``,
    ``dweight[:, w] = sum g * x[l-(W-1)+w]``, ``dx[j] = sum_w weight[:, w] * g[j+W-1-w]``,
    plus ``dfinal_states`` routed to the history positions it was copied from.
    dx is in x's dtype, dweight/dbias in the parameter dtypes, dinitial in the
    initial-states dtype (``cpp_functions.py:153-165``).
    """
    xf = to_f32(x, x_dtype)
    wf = to_f32(weight, w_dtype)
    bf = to_f32(bias, b_dtype or w_dtype) if bias is not None else None
    init_f = to_f32(initial_states, i_dtype or x_dtype) if initial_states is not None else None
    gf = to_f32(dout, x_dtype)
    b, d, seqlen = xf.shape
    width = wf.shape[1]
    masks, out_mask = _tap_masks(seq_idx, width, seqlen)
    xe = _extended_input(xf, width, init_f)
    p = _preact(xe, wf, bf, masks, out_mask, seqlen)
    if silu:
        s = _sigmoid(p)
        g = gf * (s * (np.float32(1.0) + p * (np.float32(1.0) - s)))
    else:
        g = gf
    if out_mask is not None:
        g = g * out_mask[:, None, :]
    g = g.astype(np.float32)
    dbias = g.sum(axis=(0, 2), dtype=np.float64).astype(np.float32)
    dxe = np.zeros_like(xe)
    dweight = np.zeros((d, width), np.float32)
    for w in range(width):
        gm = g if masks[w] is None else g * masks[w][:, None, :]
        dweight[:, w] = (gm * xe[:, :, w : w + seqlen]).sum(axis=(0, 2), dtype=np.float64)
        dxe[:, :, w : w + seqlen] += gm * wf[None, :, w, None]
    if dfinal_states is not None:
        df = to_f32(dfinal_states, dfinal_dtype or x_dtype)
        for k in range(width - 1):
            pos = seqlen - (width - 1) + k  # history position of final_states[..., k]
            if pos >= 0 or init_f is not None:
                dxe[:, :, pos + width - 1] += df[:, :, k]
    dx = from_f32(dxe[:, :, width - 1 :], x_dtype)
    dinit = None
    if init_f is not None:
        dinit = from_f32(dxe[:, :, : width - 1], i_dtype or x_dtype)
    return (
        dx,
        from_f32(dweight, w_dtype),
        from_f32(dbias, b_dtype or w_dtype) if bias is not None else None,
        dinit,
    )


# ----------------------------------------------------------------------------- update
def update(x, x_dtype, conv_state, weight, w_dtype, bias=None, b_dtype=None, silu=False,
           cache_seqlens=None, conv_state_indices=None):
    """Decode/speculative state update; returns ``(out, new_conv_state)``.

    Restates ``causal_conv1d_interface.py:208-245`` (``causal_conv1d_update_ref``), the
    batch-gather / padding semantics of ``cpp_functions.py:195-236`` and the update kernel
    ``cutedsl_kernels.py:436-493``:

    * the window is ``[state history | x]``; outputs use the *old* state;
    * linear mode: the state becomes the last ``state_len`` entries of ``[state | x]``;
    * circular mode (``cache_seqlens``): history is read at
      ``(cache_seqlens[b] - (W-1) + i) mod state_len`` and ``x[t]`` is written at
      ``(cache_seqlens[b] + t) mod state_len`` in order, so the last write wins;
    * ``conv_state_indices[b]`` selects the state row; a negative index gives a zero
      output row and leaves every state row untouched.
    ``cache_seqlens`` is indexed by the batch row (``cutedsl_kernels.py:449``).
    ``x`` is ``(batch, dim, seqlen)``; the state has x's storage dtype.
    """
    xf = to_f32(x, x_dtype)
    wf = to_f32(weight, w_dtype)
    bf = to_f32(bias, b_dtype or w_dtype) if bias is not None else None
    state = np.array(conv_state, copy=True)
    batch, dim, seqlen = xf.shape
    width = wf.shape[1]
    state_len = state.shape[2]
    acc = np.zeros((batch, dim, seqlen), np.float32)
    valid = np.ones(batch, bool)
    for bi in range(batch):
        row = bi if conv_state_indices is None else int(conv_state_indices[bi])
        if row < 0:
            valid[bi] = False
            continue
        st = state[row]
        if cache_seqlens is None:
            hist = st[:, state_len - (width - 1) :].copy()
            combined = np.concatenate([st, np.asarray(x[bi])], axis=1)
            state[row] = combined[:, combined.shape[1] - state_len :]
        else:
            cs = int(cache_seqlens[bi])
            idx = np.mod(cs - (width - 1) + np.arange(width - 1), state_len)
            hist = st[:, idx].copy()
            for t in range(seqlen):
                state[row][:, (cs + t) % state_len] = x[bi][:, t]
        window = np.concatenate([to_f32(hist, x_dtype), xf[bi]], axis=1)
        a = np.zeros((dim, seqlen), np.float32)
        if bf is not None:
            a = a + bf[:, None]
        for w in range(width):
            a = a + window[:, w : w + seqlen] * wf[:, w, None]
        acc[bi] = a
    if silu:
        acc = _silu(acc)
    acc[~valid] = 0.0
    return from_f32(acc, x_dtype), state


# ----------------------------------------------------------------------- varlen states
def varlen_states(x, cu_seqlens, state_len):
    """Gather the last ``state_len`` tokens of each packed sequence.

    Restates ``causal_conv1d_varlen.py:14-26`` and ``cutedsl_kernels.py:596-621``:
    ``states[b, :, s] = x[cu[b+1] - S + s]`` when that token is ``>= cu[b]``, else 0.
    ``x`` is ``(total_tokens, dim)`` in storage form; returns ``(batch, dim, S)`` whose
    memory is ``(batch, S, dim)`` (a transposed view), like the reference.
    A zero-length sequence yields an all-zero row (the kernel's behaviour; the
    reference's Python loop cannot express it).
    """
    x = np.asarray(x)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    batch = cu.shape[0] - 1
    states = np.zeros((batch, state_len, x.shape[1]), dtype=x.dtype)
    for b in range(batch):
        end = int(cu[b + 1])
        start = max(int(cu[b]), end - state_len)
        n = end - start
        if n > 0:
            states[b, state_len - n :, :] = x[start:end]
    return states.transpose(0, 2, 1)
