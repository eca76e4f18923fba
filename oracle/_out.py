"""Output dtype of the oracle functions (test infrastructure only).

The reference's torch functions return their results in the inputs' dtype
(bf16 in, bf16 out), and so does this oracle by default: that is what the
golden pins compare.  Parity of a bf16 kernel output is stated against the
fp32 value before that final rounding, so inside ``fp32_outputs()`` every
oracle function returns its result unrounded, in fp32.  Only the final
output cast is affected; intermediate roundings the reference performs (for
example the bf16 q/k of the in-kernel L2 norm) stay as they are.
"""

import contextlib

import torch

_fp32 = False


def out(t, dtype):
    """``t`` in ``dtype`` (the reference's output cast), or in fp32 inside
    ``fp32_outputs()``."""
    return t.to(torch.float32) if _fp32 else t.to(dtype)


@contextlib.contextmanager
def fp32_outputs():
    global _fp32
    prev, _fp32 = _fp32, True
    try:
        yield
    finally:
        _fp32 = prev
