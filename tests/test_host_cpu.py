"""Host-side behaviour that needs no GPU: argument errors and the deterministic-mode
selector (reference tests/test_cutedsl_backward.py:329-368)."""

import pytest
import torch

import causal_conv1d
from causal_conv1d import causal_conv1d_fn, causal_conv1d_update, cpp_functions
from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states


@pytest.mark.parametrize(
    ("env_value", "torch_deterministic", "expected"),
    [(None, False, False), (None, True, True), ("1", False, True), ("0", True, False),
     ("invalid", False, False), ("invalid", True, True)],
)
def test_deterministic_selector(env_value, torch_deterministic, expected, monkeypatch):
    if env_value is None:
        monkeypatch.delenv("CAUSAL_CONV1D_DETERMINISTIC", raising=False)
    else:
        monkeypatch.setenv("CAUSAL_CONV1D_DETERMINISTIC", env_value)
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(torch_deterministic)
    try:
        assert cpp_functions._use_deterministic_mode() is expected
    finally:
        torch.use_deterministic_algorithms(prev)


def test_version_and_exports():
    assert causal_conv1d.__version__.startswith("1.6.2")
    from causal_conv1d.causal_conv1d_interface import (  # noqa: F401
        CausalConv1dFn, causal_conv1d_ref, causal_conv1d_update_ref)
    from causal_conv1d.causal_conv1d_varlen import causal_conv1d_varlen_states_ref  # noqa: F401


def test_bad_activation_raises_not_implemented():
    x = torch.randn(1, 8, 4)
    w = torch.randn(8, 4)
    with pytest.raises(NotImplementedError):
        causal_conv1d_fn(x, w, activation="relu")
    with pytest.raises(NotImplementedError):
        causal_conv1d_update(x, torch.randn(1, 8, 3), w, activation="gelu")


def test_seq_idx_with_states_asserts():
    x = torch.randn(1, 8, 4).transpose(1, 2).contiguous().transpose(1, 2)
    w = torch.randn(8, 4)
    seq = torch.zeros(1, 4, dtype=torch.int32)
    with pytest.raises(AssertionError):
        causal_conv1d_fn(x, w, seq_idx=seq, initial_states=torch.randn(1, 8, 3))
    with pytest.raises(AssertionError):
        causal_conv1d_fn(x, w, seq_idx=seq, return_final_states=True)
    with pytest.raises(AssertionError):
        causal_conv1d_fn(torch.randn(1, 8, 4), w, return_final_states=True)  # not channel-last


def test_no_cpu_fallback():
    x = torch.randn(1, 8, 4)
    w = torch.randn(8, 4)
    with pytest.raises(ValueError, match="CUDA"):
        causal_conv1d_fn(x, w)
    with pytest.raises(ValueError, match="width"):
        causal_conv1d_fn(x, torch.randn(8, 5))
    with pytest.raises(ValueError):
        causal_conv1d_update(x, torch.randn(1, 8, 2), w)  # state_len < width - 1
    with pytest.raises(TypeError):
        causal_conv1d_varlen_states(torch.randn(10, 8), torch.tensor([0.0, 10.0]), 3)
    with pytest.raises(ValueError):
        causal_conv1d_varlen_states(torch.randn(8, 10).t(), torch.tensor([0, 10]), 3)
