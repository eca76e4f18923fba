"""ctypes binding of ``libxops_b200.so`` (the C ABI declared in
``include/xops_b200.h``).  The library is loaded from the package directory;
if it is missing the import of any op fails loudly -- there is no fallback."""

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libxops_b200.so")

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = range(5)
F32, BF16, F16 = 0, 1, 2

_p, _i64, _i32, _f, _int = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_int

# name -> argument types (restype int unless listed in _RESTYPES)
SIGNATURES = {
    "xops_last_error": [],
    "xops_version": [],
    "xops_launch_count": [],
    "xops_l2norm_last_dim": [_p, _p, _i64, _i64, _f, _int, _p],
    "xops_layer_norm_fwd": [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f,
                            _int, _int, _int, _int, _p],
    "xops_gemma_rms_norm": [_p, _p, _p, _p, _i64, _i64, _f, _int, _int, _p],
    "xops_split_rmsnorm_rope": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                _i64, _f, _int, _int, _int, _p],
    "xops_rope_inplace": [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _p],
    "xops_causal_conv1d_update": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _i64, _int, _i32, _int, _p],
    "xops_causal_conv1d_varlen": [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int,
                                  _i32, _int, _p],
    "xops_causal_conv1d_varlen_qk_l2norm": [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                            _i64, _int, _i32, _int, _i64, _f, _p],
    "xops_causal_conv1d_update_v2_slots": [_p, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _p, _i64,
                                           _i64, _i64, _i64, _i64, _int, _i32, _int, _p],
    "xops_fused_recurrent_gated_delta_rule": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                              _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                              _i64, _f, _int, _p],
    "xops_fused_sigmoid_gating_delta_rule_update": [_p, _p, _p, _f, _f, _p, _p, _p, _p, _p, _p,
                                                    _p, _p, _f, _i64, _i64, _i64, _i64, _i64,
                                                    _i64, _i64, _int, _int, _p],
    "xops_fused_qkvzba_split_reshape_cat": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                            _i64, _int, _int, _p],
    "xops_fused_gdn_gating": [_p, _p, _p, _p, _p, _p, _i64, _i64, _int, _int, _f, _f, _p],
    "xops_chunk_gated_delta_rule": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _f, _int, _p, _i64, _p],
    "xops_chunk_gated_delta_rule_gated": [_p, _p, _p, _p, _p, _p, _p, _int, _int, _i64, _int, _f,
                                          _f, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                          _i64, _i64, _i64, _i64, _f, _int, _p, _i64, _p],
    "xops_chunk_gated_delta_rule_out_norm": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                             _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f,
                                             _int, _p, _i64, _p, _int, _f, _p, _p, _i64, _p],
    "xops_chunk_gated_delta_rule_gated_out_norm": [_p, _p, _p, _p, _p, _p, _p, _int, _int, _i64,
                                                   _int, _f, _f, _p, _p, _p, _p, _i64, _i64, _i64,
                                                   _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f,
                                                   _int, _p, _i64, _i64, _i64, _p, _int, _f, _p,
                                                   _p, _i64, _p],
    "xops_causal_conv1d_varlen_qkvz": [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                       _i64, _i64, _int, _i32, _int, _int, _f, _p],
    "xops_chunk_gated_delta_rule_workspace_size": [_i64, _i64, _i64, _i64, _i64, _i64, _int, _int],
    "xops_chunk_gated_delta_rule_noalloc": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                            _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f, _int,
                                            _p],
    "xops_chunk_local_cumsum": [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    "xops_chunk_scaled_dot_kkt_fwd": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _p],
    "xops_solve_tril": [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _p],
    "xops_recompute_w_u_fwd": [_p, _p, _p, _p, _p, _int, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                               _i64, _i64, _p],
    "xops_chunk_gated_delta_rule_fwd_h": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                          _i64, _i64, _i64, _i64, _i64, _p],
    "xops_chunk_fwd_o": [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                         _i64, _f, _p],
    "xops_total_chunks": [_p, _i64, _i64, _i64, _i64],
    "xops_device_error_count": [],
}
_RESTYPES = {"xops_last_error": C.c_char_p, "xops_version": C.c_char_p,
             "xops_launch_count": C.c_uint64, "xops_total_chunks": C.c_int64,
             "xops_chunk_gated_delta_rule_workspace_size": C.c_int64}

_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the CDLL with typed entry points."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m torch_npu_ops_b200.build` "
                    "(the CUDA kernels are required; there is no CPU fallback)")
            lib = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = lib
    return _lib


class XopsError(RuntimeError):
    """Raised when a C-ABI call returns a non-zero status."""

    def __init__(self, status, msg):
        super().__init__(msg)
        self.status = status


def call(name, *args):
    """Call an entry point; raise XopsError (a RuntimeError, like the
    reference's TORCH_CHECK failures) on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.xops_last_error().decode(errors="replace")
        raise XopsError(rc, f"{name}: {msg} (status {rc})")
    return rc


def launch_count():
    return int(load().xops_launch_count())
