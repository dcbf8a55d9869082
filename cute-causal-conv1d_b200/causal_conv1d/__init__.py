"""causal_conv1d for NVIDIA B200 (sm_100a): depthwise causal conv1d kernels.

Drop-in for the public API of causal-conv1d 1.6.2 (Butterfingrz/cute-causal-conv1d):
``causal_conv1d_fn``, ``causal_conv1d_update`` and
``causal_conv1d.causal_conv1d_varlen.causal_conv1d_varlen_states``, backed by
hand-written CUDA kernels reached through the C ABI of ``libcc1d_b200.so``.
"""

__version__ = "1.6.2.post1+b200"

from causal_conv1d.causal_conv1d_interface import causal_conv1d_fn, causal_conv1d_update  # noqa: E402,F401
from causal_conv1d import torch_ops  # noqa: E402,F401  (registers torch.ops.causal_conv1d.*)
