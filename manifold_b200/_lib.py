"""ctypes binding of libgfn_b200.so (the C ABI declared in include/gfn_b200.h).

The library is built in-tree (``manifold_b200/libgfn_b200.so``) by
``manifold_b200.build.build()``.  There is no fallback: if the library is
missing or a call fails, a ``GfnError`` is raised.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("GFN_B200_LIB") or os.path.join(_HERE, "libgfn_b200.so")

_c_float_p = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_p = ctypes.c_void_p

# name -> argtypes (all return int unless listed in _RESTYPES)
_SIGS = {
    "gfn_status_string": [_i],
    "gfn_last_error_message": [],
    "gfn_build_info": [],
    "gfn_get_device_error": [_p, _i, _p],
    "gfn_christoffel_fused": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _f, _f, _f, _i, _f, _f, _p],
    "gfn_leapfrog_fused": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _f, _p, _i, _i, _i, _i, _i, _i, _f,
                           _f, _f, _p],
    "gfn_leapfrog_sequence_forward": [_p, _p, _ll, _p, _p, _p, _p, _ll, _p, _p, _ll, _i, _i, _i,
                                      _i, _i, _i, _f, _p, _p, _p, _p, _p],
    "gfn_leapfrog_pack_floats": [_i, _i, _i, _i],
    "gfn_leapfrog_pack": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p, _ll, _p],
    "gfn_leapfrog_plan": [_i, _i, _i, _i, _i, _p],
    "gfn_debug_set_phase_profile": [_p],
    "gfn_debug_latency_probe": [_i, _i, _i, _p, _p],
    "gfn_parallel_scan_workspace_floats": [_i, _i, _i],
    "gfn_leapfrog_pack_train_floats": [_i, _i, _i, _i],
    "gfn_leapfrog_pack_train": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p, _ll,
                                _p],
    "gfn_leapfrog_sequence_forward_train": [_p, _p, _ll, _p, _p, _p, _p, _ll, _p, _p, _ll, _i, _i,
                                            _i, _i, _i, _i, _f, _p, _p, _p, _p, _p, _p],
    "gfn_leapfrog_backward_workspace_floats": [_i, _i, _i, _i, _i, _i],
    "gfn_leapfrog_sequence_backward": [_p, _p, _p, _p, _p, _ll, _p, _p, _ll, _p, _p, _p, _p, _i, _i,
                                       _i, _i, _i, _i, _f, _p, _p, _p, _p, _ll, _p],
    "gfn_leapfrog_layered_pack_floats": [_i, _i, _i, _i],
    "gfn_leapfrog_layered_pack": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p, _ll,
                                  _p],
    "gfn_leapfrog_layered_workspace_floats": [_i, _i],
    "gfn_leapfrog_layered_set_mixing": [_i],
    "gfn_debug_layered_timing": [_i],
    "gfn_debug_head_profile": [_p],
    "gfn_debug_layered_timing_read": [_p, _p, _p],
    "gfn_leapfrog_layered_forward": [_p, _p, _ll, _p, _p, _p, _p, _ll, _p, _p, _ll, _i, _i, _i, _i,
                                     _i, _i, _f, _p, _p, _p, _p, _p, _ll, _p],
    "gfn_split_f16": [_p, _ll, _ll, _i, _i, _p, _p, _p],
    "gfn_gemm_split_f16_tc": [_i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p],
    "gfn_cross_entropy_forward": [_p, _p, _ll, _i, _ll, _p, _p, _p],
    "gfn_cross_entropy_backward": [_p, _p, _p, _ll, _i, _ll, _p, _p, _p],
    "gfn_gemm_split_f16": [_i, _i, _i, _p, _i, _p, _i, _p, _p, _f, _p, _p, _p],
    "gfn_parallel_scan": [_p, _p, _p, _p, _ll, _i, _i, _i, _p],
    "gfn_parallel_scan_noalloc": [_p, _p, _p, _i, _i, _i, _p],
    "gfn_parallel_layer_scan": [_p, _p, _p, _i, _i, _i, _i, _f, _p],
    "gfn_functional_embedding": [_p, _ll, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f, _i, _p, _p, _p],
    "gfn_leapfrog_fused_gated": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f, _p, _i, _i, _i, _i, _i,
                                 _i, _f, _f, _f, _p],
    "gfn_integrator_heads": [_i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f, _p, _i, _i, _i, _i, _i,
                             _i, _i, _f, _f, _f, _p, _p, _i, _f, _f, _p],
    "gfn_christoffel_torus": [_p, _p, _p, _i, _i, _f, _f, _p],
    "gfn_christoffel_backward_workspace_floats": [_i, _i, _i],
    "gfn_christoffel_backward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _f, _f, _f,
                                 _i, _f, _f, _p, _ll, _p],
    "gfn_leapfrog_step_backward_workspace_floats": [_i, _i, _i, _i, _i],
    "gfn_leapfrog_backward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                              _p, _i, _i, _i, _f, _p, _i, _i, _i, _f, _f, _p, _ll, _p],
}
_RESTYPES = {
    "gfn_status_string": ctypes.c_char_p,
    "gfn_last_error_message": ctypes.c_char_p,
    "gfn_build_info": ctypes.c_char_p,
    "gfn_leapfrog_pack_floats": ctypes.c_longlong,
    "gfn_parallel_scan_workspace_floats": ctypes.c_longlong,
    "gfn_leapfrog_pack_train_floats": ctypes.c_longlong,
    "gfn_leapfrog_backward_workspace_floats": ctypes.c_longlong,
    "gfn_leapfrog_layered_pack_floats": ctypes.c_longlong,
    "gfn_leapfrog_layered_workspace_floats": ctypes.c_longlong,
    "gfn_christoffel_backward_workspace_floats": ctypes.c_longlong,
    "gfn_leapfrog_step_backward_workspace_floats": ctypes.c_longlong,
}

EXPORTED = tuple(_SIGS)


class GfnError(RuntimeError):
    pass


_lib = None


def load():
    """Load the shared library (once).  Raises GfnError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise GfnError(f"{LIB_PATH} is missing; build it with manifold_b200.build.build()")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = lib
    return lib


def check(status, what):
    if status != 0:
        lib = load()
        msg = lib.gfn_last_error_message().decode()
        kind = lib.gfn_status_string(status).decode()
        raise GfnError(f"{what}: {kind} ({status}): {msg}")


def call(name, *args):
    fn = getattr(load(), name)
    check(fn(*args), name)


def ptr(t):
    """Device pointer of a tensor, or None for an absent operand."""
    if t is None:
        return None
    return t.data_ptr()


def stream_of(device):
    return torch.cuda.current_stream(device).cuda_stream


def device_error(reset=True, device=None):
    bits = ctypes.c_int(0)
    call("gfn_get_device_error", ctypes.byref(bits), 1 if reset else 0,
         stream_of(device) if device is not None else torch.cuda.current_stream().cuda_stream)
    return bits.value


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise GfnError("manifold_b200 runs on CUDA tensors only (no CPU path); got a "
                           f"{t.device} tensor")
