"""ctypes binding of the C ABI in include/viktor_b200.h (libviktor_b200.so, built in-tree).

There is no fallback: if the library is missing or a call returns a non-zero status, the call raises.
"""

from __future__ import annotations

import ctypes as C
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libviktor_b200.so")

VK_OK, VK_ERR_ARG, VK_ERR_CUDA, VK_ERR_UNSUPPORTED = 0, -1, -2, -3
_STATUS = {VK_ERR_ARG: "bad argument", VK_ERR_CUDA: "CUDA error", VK_ERR_UNSUPPORTED: "unsupported geometry"}
DEVERR = {1: "wait for a TMA stage timed out", 2: "wait for a free stage timed out",
          4: "wait for the tensor-core accumulator timed out", 8: "index out of range (access skipped)"}

p, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t

_SIGS = {
    "vk_version": (i32, []),
    "vk_read_device_errors": (i32, [C.POINTER(C.c_uint32), i32]),
    "vk_set_pdl": (i32, [i32]),
    "vk_test_bounded_wait": (i32, [C.c_uint64, p, p]),
    "vk_test_noalloc_poison": (i32, [p]),
    "vk_add_rmsnorm": (i32, [p, p, p, p, i64, i32, f32, p]),
    "vk_embed_rmsnorm": (i32, [p, p, i64, p, p, p, i64, i32, f32, p]),
    "vk_qkv_rope_cache": (i32, [p, p, p, p, p, i32, p, p, p, p, p, p, p, p, i64, i64, i64, i32, i32, f32, i32, i32,
                                i32, p]),
    "vk_linear": (i32, [p, p, p, i64, i32, i32, i32, i32, p]),
    "vk_swiglu": (i32, [p, p, i64, i32, p]),
    "vk_greedy_update": (i32, [p, i64, p, p, p, i32, p, p, p, p, p, p, i64, i64, p, p, p, i32, i32, i32, i32, p, p,
                               p, p]),
    "vk_head_select": (i32, [p, p, f32, p, p, p, p, i32, p, p, p, p, p, p, i64, i64, p, p, p, i32, i32, i32, i32, p, p, p,
                             p, i64, f32, p, i32, p]),
    "vk_prefill_plan": (i32, [p, i32, i32, i32, i64, p, p, p, p, p, p, p, p]),
    "vk_sample_update": (i32, [p, i64, p, p, p, i32, p, p, p, p, p, p, i64, i64, p, p, p, i32, i32, i32, i32, p, p,
                               p, p, i64, f32, p]),
    "vk_decode_attention_workspace_bytes": (sz, [i32, i32]),
    "vk_decode_attention": (i32, [p, p, p, p, p, i32, i32, i32, i32, i64, i64, p, sz, p]),
    "vk_kv_quantize": (i32, [p, p, i32, i32, i64, i64, p, i32, i32, p, p, p, p, i32, p]),
    "vk_decode_attention_i8_workspace_bytes": (sz, [i32, i32, i32]),
    "vk_decode_attention_i8": (i32, [p, p, p, p, p, p, p, p, p, p, i32, i32, i32, i32, i64, i64, i32, i32, p, sz,
                                     p]),
    "vk_align": (i32, [p, i32, p, i32, i32, i32, p, p, i32]),
    "vk_overlap_cut": (i32, [p, i32, p, i32, i32, C.c_double, p]),
    "vk_stitch": (i32, [p, p, p, i32, i32, p, i64, p]),
    "vk_decode_attention_noalloc": (i32, [p, p, p, p, p, i32, i32, i32, i32, i64, i64, p]),
    "vk_prefill_attention": (i32, [p, p, p, p, i32, i32, i64, i32, i32, i32, i64, i64, p, p]),
    "vk_linear_rmsnorm": (i32, [p, p, f32, p, p, i64, i32, i32, i32, i32, p]),
    "vk_linear_qkv_rope_cache": (i32, [p, p, f32, p, p, p, p, p, i32, p, p, p, p, p, p, p, p, i64, i64, i64, i32, i32,
                                       f32, i32, i32, p]),
    "vk_linear_residual": (i32, [p, p, p, p, i64, i32, p]),
    "vk_linear_add_rmsnorm": (i32, [p, p, p, p, p, p, i64, i32, f32, p]),
    "vk_row_ssq": (i32, [p, p, i64, i32, p]),
    "vk_ssq_rmsnorm": (i32, [p, p, p, p, i64, i32, f32, p]),
    "vk_fold_norm_weight": (i32, [p, p, p, i64, i32, p]),
    "vk_linear_bias_act": (i32, [p, p, p, p, i64, p, i64, i32, i32, i32, p]),
    "vk_cast_f32_bf16": (i32, [p, p, i64, p]),
    "vk_gather_rows": (i32, [p, p, p, i64, i32, i64, p]),
    "vk_copy_rows": (i32, [p, p, i64, p, p, i64, i64, i32, p]),
    "vk_scatter_embed": (i32, [p, p, i64, i64, p, i64, i32, p]),
}

_lib = None
_HOST_ONLY = {"vk_version", "vk_read_device_errors", "vk_set_pdl", "vk_decode_attention_workspace_bytes",
              "vk_decode_attention_i8_workspace_bytes", "vk_align", "vk_overlap_cut", "vk_stitch"}
launches = 0  # kernels launched through call() (each launching entry point launches exactly one kernel)


def lib_path() -> str:
    return _LIB_PATH


def load():
    """Loads the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"viktor_b200 CUDA library not built ({_LIB_PATH}); run python -m viktor_b200.build")
        lib = C.CDLL(_LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def call(name: str, *args):
    """Calls an entry point and raises RuntimeError on a non-zero status."""
    global launches
    rc = getattr(load(), name)(*args)
    if rc != VK_OK:
        raise RuntimeError(f"{name} failed: {_STATUS.get(rc, rc)}")
    if name not in _HOST_ONLY:
        launches += 1
    return rc


def read_device_errors(clear: bool = True) -> int:
    bits = C.c_uint32(0)
    call("vk_read_device_errors", C.byref(bits), 1 if clear else 0)
    return bits.value


def check_device_errors():
    """Raises if any kernel flagged an error since the last check."""
    bits = read_device_errors(clear=True)
    if bits:
        msgs = [m for b, m in DEVERR.items() if bits & b]
        raise RuntimeError("viktor_b200 kernel error: " + "; ".join(msgs))


def set_pdl(enable: bool):
    call("vk_set_pdl", 1 if enable else 0)
