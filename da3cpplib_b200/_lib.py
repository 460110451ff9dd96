"""ctypes binding of libda3b.so (the native library built in-tree by build.py).

The library is the product: every compute call goes through it. If it is missing
the import raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libda3b.so")

_lib = None

c_int = ctypes.c_int
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p
c_char_p = ctypes.c_char_p
c_size_t = ctypes.c_size_t

# name -> (restype, argtypes); one entry per symbol of include/da3b.h and include/da3cpp/da3_c.h
SIGNATURES = {
    "da3b_abi_version": (c_int, []),
    "da3b_device_status": (c_int, []),
    "da3b_dequant_q8_0": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "da3b_linear_f16": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int,
                                c_void_p, c_int, c_void_p]),
    "da3b_linear_resid_f32": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p, c_int, c_void_p]),
    "da3b_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "da3b_quantize_q8_0": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_repack_q8_0": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_linear_q8q8_i8": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                    c_int, c_void_p]),
    "da3b_debug_wait_timeout": (c_int, [ctypes.c_ulonglong, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_debug_mma_cycles": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "da3b_set_attention_split": (c_int, [c_int]),
    "da3b_linear_tiles": (c_int, [c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "da3b_repack_q8_0_planar": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "da3b_dequant_q8p": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "da3b_linear_q8p_f16": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                    c_void_p]),
    "da3b_linear_q8p_resid_f32": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                          c_void_p, c_int, c_void_p]),
    "da3b_transpose_v": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
    "da3b_attention_vt": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "da3b_attention_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_upsample_nhwc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p]),
    "da3b_output_conv2": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_void_p, c_float, c_void_p, c_int, c_void_p]),
    "da3b_resize_u8": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p]),
    "da3b_preprocess_legacy": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                       ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_void_p]),
    "da3b_patchify": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "da3b_pack_conv_weight": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "da3b_conv_nhwc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p,
                               c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_load": (c_void_p, [c_char_p, c_int]),
    "da3b_processed_size": (c_int, [c_void_p, c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int)]),
    "da3b_infer_device": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                  c_void_p]),
    "da3b_infer_host": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_infer_prepared": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_last_pose": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "da3b_last_sky": (c_int, [c_void_p, c_int, c_void_p]),
    "da3b_ray_pose": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                              c_void_p, c_void_p]),
    "da3b_nested_align": (ctypes.c_float, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_int64,
                                           c_void_p, c_void_p]),
    "da3b_ref_views": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int]),
    "da3b_launches": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int]),
    "da3b_debug_feature": (c_int, [c_void_p, c_int, c_void_p, c_size_t, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "da3b_set_capture_residuals": (c_int, [c_void_p, c_int]),
    "da3b_debug_residual": (c_int, [c_void_p, c_int, c_void_p, c_size_t, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "da3b_set_graphs": (c_int, [c_void_p, c_int]),
    "da3b_set_raw_logits": (c_int, [c_void_p, c_int]),
    "da3b_set_act_quant": (c_int, [c_void_p, c_int]),
    "da3b_model_dims": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    # reference-compatible C ABI (include/da3cpp/da3_c.h)
    "da_capi_abi_version": (c_int, []),
    "da_capi_load": (c_void_p, [c_char_p, c_int]),
    "da_capi_load_nested": (c_void_p, [c_char_p, c_char_p, c_int]),
    "da_capi_free": (None, [c_void_p]),
    "da_capi_info_json": (c_void_p, [c_void_p]),
    "da_capi_free_string": (None, [c_void_p]),
    "da_capi_last_error": (c_char_p, [c_void_p]),
    "da_capi_depth_path": (c_void_p, [c_void_p, c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "da_capi_pose_path": (c_int, [c_void_p, c_char_p, c_void_p, c_void_p]),
    "da_capi_depth_pose_multi": (c_void_p, [c_void_p, ctypes.POINTER(c_char_p), c_int, ctypes.POINTER(c_int),
                                            ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_void_p, c_void_p]),
    "da_capi_depth_dense": (c_int, [c_void_p, c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_void_p, ctypes.POINTER(c_int)]),
    "da_capi_points": (c_int, [c_void_p, c_char_p, c_float, ctypes.POINTER(c_int), c_void_p, c_void_p]),
    "da_capi_export_glb": (c_int, [c_void_p, c_char_p, c_char_p]),
    "da_capi_export_colmap": (c_int, [c_void_p, c_char_p, c_char_p, c_int]),
    "da_capi_free_floats": (None, [c_void_p]),
    "da_capi_free_bytes": (None, [c_void_p]),
}


def load() -> ctypes.CDLL:
    """Load libda3b.so (raises OSError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"libda3b.so not built at {LIB_PATH}; run `python da3cpplib_b200/build.py`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with status {rc}")
