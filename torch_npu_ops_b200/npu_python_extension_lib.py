"""The pybind module's schemas (npu_python_extension/op_register.cpp:52-63):
``gemma_rms_norm(x, gamma, epsilon) -> (rstd, y)`` and
``layer_norm_fwd(x, weight, bias, eps, z, group_size, norm_before_gate,
is_rms_norm) -> y``, backed by the CUDA kernels."""

from .ops import npu_gemma_rms_norm as _gemma
from .ops import layer_norm_fwd as _ln


def gemma_rms_norm(x, gamma, epsilon):
    return _gemma(x, gamma, epsilon)


def layer_norm_fwd(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm):
    return _ln(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm)
