"""ctypes binding of libonnxsharp_cuda (the C ABI declared in include/onnxsharp_cuda.h).

The library is loaded from the package directory (built in-tree by
``onnxsharp_b200.build``). There is no fallback: if the shared object is
missing or fails to load, every call raises :class:`OscUnavailable`.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libonnxsharp_cuda.so"

# status codes (enum osc_status)
OSC_OK = 0
OSC_EINVAL = 1
OSC_ENOMEM = 2
OSC_ECUDA = 3
OSC_ENCCL = 4
OSC_ETIMEDOUT = 5
OSC_EFAULT_INJECTED = 6
OSC_EUNSUPPORTED = 7

STATUS_NAMES = {
    OSC_OK: "OSC_OK", OSC_EINVAL: "OSC_EINVAL", OSC_ENOMEM: "OSC_ENOMEM", OSC_ECUDA: "OSC_ECUDA",
    OSC_ENCCL: "OSC_ENCCL", OSC_ETIMEDOUT: "OSC_ETIMEDOUT", OSC_EFAULT_INJECTED: "OSC_EFAULT_INJECTED",
    OSC_EUNSUPPORTED: "OSC_EUNSUPPORTED",
}

# activation codes (enum osc_act)
ACT_NONE, ACT_SILU, ACT_RELU, ACT_SIGMOID = 0, 1, 2, 3
ACT_FAST = 16  # OR into conv2d_direct's activation: hardware ex2/rcp Sigmoid/SiLU


class OscError(RuntimeError):
    """A non-zero status returned by the C ABI (mirrors OnnxSharpException)."""

    def __init__(self, status: int, message: str, call: str):
        self.status = status
        self.call = call
        super().__init__(f"{call}: {STATUS_NAMES.get(status, status)}: {message}")


class OscUnavailable(RuntimeError):
    """The CUDA library could not be loaded (not built, or no CUDA driver)."""


vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong
f32 = C.c_float
sz = C.c_size_t
pp = C.POINTER(C.c_void_p)

# name -> (restype, argtypes). Kept in the order of include/onnxsharp_cuda.h.
SIGNATURES: dict[str, tuple] = {
    "osc_version": (i32, []),
    "osc_last_error": (C.c_char_p, []),
    "osc_create": (i32, [i32, pp]),
    "osc_destroy": (i32, [vp]),
    "osc_set_stream": (i32, [vp, vp]),
    "osc_get_stream": (vp, [vp]),
    "osc_own_stream": (vp, [vp]),
    "osc_synchronize": (i32, [vp, i32]),
    "osc_reserve_scratch": (i32, [vp, sz]),
    "osc_profile_enable": (i32, [vp, i32]),
    "osc_profile_read": (i32, [vp, C.c_char_p, C.POINTER(C.c_double), C.POINTER(i32)]),
    "osc_profile_reset": (i32, [vp]),
    "osc_launch_count": (C.c_ulonglong, [vp]),
    "osc_selfcheck_recip": (i32, [vp, C.POINTER(C.c_ulonglong), C.POINTER(C.c_uint)]),
    "osc_selfcheck_fast_act": (i32, [vp, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "osc_selfcheck_timeout": (i32, [vp, i32]),
    "osc_dynamic_quantize_linear_f32": (i32, [vp, vp, i64, vp, vp, vp]),
    "osc_letterbox_u8": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, C.POINTER(i32)]),
    "osc_letterbox_batch_u8": (i32, [vp, vp, i32, i64, i32, i32, i32, i32, i32, i32, i32, vp, i64, C.POINTER(i32)]),
    "osc_yolo_detect_f32": (i32, [vp, vp, i32, i32, i32, C.c_float, C.c_float, i32, i32, i32, vp, vp, vp]),
    "osc_matmul_batched_f32": (i32, [vp, i32, i32, i32, i32, i32, vp, i64, i64, i64, i64, vp, i64, i64, i64, i64, vp,
                                     vp]),
    "osc_gemm_onnx_f32": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, i32, C.c_float, C.c_float, vp, i64, vp]),
    "osc_matmul_integer_i8": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp]),
    "osc_graph_begin": (i32, [vp]),
    "osc_graph_end": (i32, [vp, pp]),
    "osc_graph_launch": (i32, [vp, vp]),
    "osc_graph_free": (i32, [vp]),
    "osc_group_create": (i32, [i32, C.POINTER(i32), pp]),
    "osc_group_destroy": (i32, [vp]),
    "osc_group_size": (i32, [vp, C.POINTER(i32)]),
    "osc_group_ctx": (i32, [vp, i32, pp]),
    "osc_group_synchronize": (i32, [vp, i32]),
    "osc_group_allgather": (i32, [vp, pp, pp, sz]),
    "osc_group_allreduce_minmax": (i32, [vp, pp]),
    "osc_group_run_sharded": (i32, [vp, pp, pp, pp, sz]),
    "osc_plan_build": (i32, [vp, vp, pp]),
    "osc_plan_run": (i32, [vp, vp, vp]),
    "osc_plan_arena_bytes": (i32, [vp, C.POINTER(sz)]),
    "osc_plan_buffer": (i32, [vp, i32, vp, pp, C.POINTER(i64)]),
    "osc_plan_free": (i32, [vp]),
    "osc_arena_assign": (i32, [i32, vp, vp, vp, vp, C.POINTER(sz)]),
    "osc_malloc": (i32, [vp, sz, pp]),
    "osc_free": (i32, [vp, vp]),
    "osc_memcpy_htod": (i32, [vp, vp, vp, sz]),
    "osc_memcpy_dtoh": (i32, [vp, vp, vp, sz]),
    # MatMul + FusedBias
    "osc_gemm_prepack_f32": (i32, [vp, vp, i32, i32, i32, pp]),
    "osc_gemm_prepack_f32_host": (i32, [vp, vp, i32, i32, i32, pp]),
    "osc_gemm_weights_free": (i32, [vp]),
    "osc_gemm_bias_f32": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp, i32]),
    "osc_gemm_bias_f32_noalloc": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp, i32]),
    "osc_gemm_split_a_f32": (i32, [vp, vp, i32, i32, i32, i32, vp, vp]),
    "osc_gemm_bias_presplit_f32": (i32, [vp, vp, vp, i32, i32, vp, vp, i32, vp, i32]),
    # Conv + FusedActivation
    "osc_conv_prepack_f32": (i32, [vp, vp, i32, i32, i32, i32, i32, pp]),
    "osc_conv_weights_free": (i32, [vp]),
    "osc_conv2d_bias_act_f32": (i32, [vp, vp, i32, i32, i32, i32, vp] + [i32] * 9 + [vp, i32, vp, i32, i32]),
    # DynamicQuantizeMatMul
    "osc_dqmm_prepack": (i32, [vp, vp, i32, i32, i32, vp, i32, i32, pp]),
    "osc_dqmm_weights_free": (i32, [vp]),
    "osc_dqmm_f32": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp, vp, vp, vp, vp, vp]),
    "osc_dqmm_shard_f32": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp, vp, vp, i32, i32, vp, vp, vp]),
    "osc_minmax_f32": (i32, [vp, vp, C.c_long, vp]),
    # FusedAttention
    "osc_attention_f32": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, i32, vp]),
    # graph glue
    "osc_conv2d_ex_f32": (i32, [vp, vp, i64, i32, i32, i32, i32, vp] + [i32] * 8 + [vp, i32, vp, i64, vp, i64, i32,
                                                                                   i32]),
    "osc_conv2d_direct_f32": (i32, [vp, vp, i64, i32, i32, i32, i32, vp, i32, i32, i32] + [i32] * 9 +
                              [vp, i32, vp, i64, vp, i64, i32, i32]),
    "osc_maxpool2d_f32": (i32, [vp, vp, i64, i32, i32, i32, i32] + [i32] * 8 + [vp, i64, i32, i32]),
    "osc_resize_nearest_f32": (i32, [vp, vp, i64, i32, i32, i32, i32, i32, i32, vp, i64]),
    "osc_binary_f32": (i32, [vp, i32, vp, vp, i32, vp, vp, i32, vp]),
    "osc_unary_f32": (i32, [vp, vp, vp, i64, i32]),
    "osc_softmax_f32": (i32, [vp, vp, vp, i64, i32]),
    "osc_dfl_f32": (i32, [vp, vp, i32, i32, i32, i32, vp]),
    "osc_yolo_decode_f32": (i32, [vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "osc_layernorm_f32": (i32, [vp, vp, i32, i32, vp, vp, f32, vp]),
    "osc_psa_attention_f32": (i32, [vp, vp, i64, i32, i32, i32, i32, i32, f32, vp, i64]),
}

_lib: C.CDLL | None = None
_load_error: str | None = None


def load() -> C.CDLL:
    """Load the shared library once and attach the signatures."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise OscUnavailable(_load_error)
    path = Path(os.environ.get("OSC_LIB", LIB_PATH))
    if not path.exists():
        _load_error = f"{path} is not built (run python -m onnxsharp_b200.build)"
        raise OscUnavailable(_load_error)
    try:
        lib = C.CDLL(str(path))
    except OSError as e:  # pragma: no cover - depends on the machine
        _load_error = f"cannot load {path}: {e}"
        raise OscUnavailable(_load_error) from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().osc_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def call(name: str, *args):
    """Call an int-returning ABI function; raise OscError on a non-zero status."""
    fn = getattr(load(), name)
    st = fn(*args)
    if st != OSC_OK:
        raise OscError(st, last_error(), name)
    return st


def ptr(x) -> int | None:
    """Device or host address of a torch tensor / numpy array / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x).__name__}")
