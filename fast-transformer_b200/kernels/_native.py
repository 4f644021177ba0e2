"""ctypes binding of libfastb200.so (the C ABI declared in include/fastb200.h).

There is no fallback: if the library is missing or fails to load, importing any kernel
module raises, so a GPU run can never silently route around the CUDA kernels.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(os.path.dirname(_HERE), "libfastb200.so")

FB_OK = 0
FB_ERR_SHAPE = -2
_STATUS = {
    -1: "bad argument",
    -2: "unsupported shape",
    -3: "kernel launch failed",
    -4: "tensor-map encoder unavailable or refused the map",
    -5: "workspace too small",
    -6: "request larger than the entry point's fixed limit",
}

_c_int, _c_float, _c_size, _c_i64, _vp = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_int64, ctypes.c_void_p

# name -> (restype, argtypes)
_SIGNATURES = {
    "fb_version": (_c_int, []),
    "fb_device_error": (_c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "fb_decode_attention_ctas": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "fb_decode_attention_workspace": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "fb_decode_attention": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_size,
                                     _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp]),
    "fb_decode_attention_partials": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_size,
                                              _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp]),
    "fb_decode_attention_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                                             _c_int, _c_float, _vp]),
    "fb_decode_attention_combine": (_c_int, [_vp, _c_int, _vp, _vp, _c_size,
                                             _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "fb_verify_attention_splits": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "fb_verify_attention_workspace": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "fb_verify_attention": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_int, _c_int, _c_int, _c_int,
                                     _c_int, _c_int, _c_float, _c_int, _vp]),
    "fb_qk_norm_rope_append": (_c_int, [_vp, _c_int, _vp, _vp, _c_float, _c_float, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                        _c_int, _c_int, _vp]),
    "fb_rmsnorm": (_c_int, [_vp, _c_i64, _vp, _vp, _c_int, _c_int, _c_float, _vp]),
    "fb_add_rmsnorm": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp]),
    "fb_embed_rmsnorm": (_c_int, [_vp, _vp, _c_i64, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp]),
    "fb_swiglu": (_c_int, [_vp, _c_int, _vp, _c_int, _c_int, _vp]),
    "fb_linear_splits": (_c_int, [_c_int, _c_int, _c_int]),
    "fb_linear_finished_splits": (_c_int, [_c_int, _c_int, _c_int]),
    "fb_decode_attention_cluster_shape": (_c_int, [_c_int, _c_int]),
    "fb_linear": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "fb_allreduce_add_rmsnorm": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp,
                                          _c_int, _c_int, _c_float, _vp]),
    "fb_merge_splits": (_c_int, [_vp, _c_int, _c_i64, _vp, _c_int, _vp]),
    "fb_swiglu_blocked": (_c_int, [_vp, _c_int, _vp, _c_int, _c_int, _vp]),
    "fb_reduce_scatter_push": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "fb_allreduce_push": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "fb_allreduce_sum_add_rmsnorm": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_float,
                                              _vp]),
    "fb_prefill_attention": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float,
                                      _vp]),
    "fb_spec_propose": (_c_int, [_vp, _c_i64, _vp, _vp, _c_i64, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                 _c_int, _c_int, _c_int, _c_int, _vp]),
    "fb_spec_within_margin": (_c_int, [_vp, _c_i64, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp]),
    "fb_spec_settle": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _vp]),
    "fb_spec_relocate": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "fb_argmax_candidates_bytes": (_c_size, [_c_int, _c_int]),
    "fb_linear_argmax": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_i64, _vp, _vp]),
    "fb_argmax_candidates": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "fb_argmax_workspace": (_c_size, [_c_int, _c_i64]),
    "fb_argmax": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _c_size, _vp]),
}


def _load():
    if not os.path.exists(LIBRARY_PATH):
        raise ImportError(
            f"{LIBRARY_PATH} is not built; run `python fast-transformer_b200/build.py` "
            "(the CUDA kernels are required, there is no CPU fallback)"
        )
    lib = ctypes.CDLL(LIBRARY_PATH)
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


def exported_names():
    return sorted(_SIGNATURES)


#: Kernels each launching entry point enqueues (fb_argmax runs two stages).
_KERNELS_PER_CALL = {"fb_argmax": 2}
_NON_LAUNCHING = {"fb_device_error"}
#: Running count of libfastb200 kernels enqueued (or recorded into a graph) by this process.
launches = 0


def check(status, what):
    global launches
    if status != FB_OK:
        raise RuntimeError(f"{what}: {_STATUS.get(status, 'error')} (status {status})")
    if what not in _NON_LAUNCHING:
        launches += _KERNELS_PER_CALL.get(what, 1)


def stream():
    """The current CUDA stream as the void* the C ABI expects (the capture stream inside a graph)."""
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(tensor):
    return ctypes.c_void_p(tensor.data_ptr()) if tensor is not None else None


def device_error():
    """Reads and clears the library's device error word (synchronises the device)."""
    flags = ctypes.c_uint(0)
    check(lib.fb_device_error(ctypes.byref(flags)), "fb_device_error")
    return flags.value


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("libfastb200 kernels take CUDA tensors only (no CPU fallback)")
