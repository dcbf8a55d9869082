"""Tolerances used by the parity tests.

Kernel vs oracle (the parity bar): the benchmark's tolerance table, taking the reference test's
stricter bf16 pair (``tests/test_causal_conv1d.py:75-78`` in the reference):
fp32 3e-4/1e-3, fp16 3e-3/5e-3, bf16 1e-2/5e-2; dweight/dbias 1e-3/1e-3 for fp32
parameters, and 1e-2/5e-2 for 16-bit parameters (reference
``tests/test_cutedsl_backward.py:323-327``).  conv_state, varlen states and final states
are compared bit for bit.

Oracle vs golden vectors (pinning the CPU restatement): both sides compute in fp32 and
round once, so they may differ by accumulation order and by one rounding of the output
dtype: 2 ulp of the output dtype relative, plus a small absolute floor.
"""

PARITY = {
    "float32": (3e-4, 1e-3),
    "float16": (3e-3, 5e-3),
    "bfloat16": (1e-2, 5e-2),
}

GRAD_PARAM = {
    "float32": (1e-3, 1e-3),
    "float16": (1e-2, 5e-2),
    "bfloat16": (1e-2, 5e-2),
}

PIN = {
    "float32": (2e-5, 2e-5),
    "float16": (2.0 * 2.0 ** -10, 1e-4),
    "bfloat16": (2.0 * 2.0 ** -7, 1e-3),
}
