"""ctypes binding of the C ABI declared in include/xinfer_b200.h.

The shared library is built in-tree (xinfer_b200/libxinfer_b200.so, see xinfer_b200/build.py).
There is no fallback: importing the product path without the library raises.
"""

import ctypes
import os
from pathlib import Path

MAX_LAYERS = 64
MAX_BATCH = 8

XB_OK, XB_ERR_INVALID, XB_ERR_CUDA, XB_ERR_DEVICE, XB_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
FAMILY_QWEN3, FAMILY_QWEN35 = 1, 2
LAYER_ATTENTION, LAYER_DELTANET = 0, 1

LIBRARY_NAME = "libxinfer_b200.so"
LIBRARY_PATH = Path(__file__).resolve().parent / LIBRARY_NAME

# Every symbol the header declares (checked by the CPU test suite).
EXPORTED = (
    "xb_model_create", "xb_model_destroy", "xb_decode_workspace_bytes", "xb_workspace_init",
    "xb_decode_step", "xb_workspace_check", "xb_rope_inv_freq", "xb_last_error",
    "xb_abi_version", "xb_decode_step_static", "xb_debug_trace", "xb_debug_fault",
    "xb_prefix_attention", "xb_prefill_workspace_bytes", "xb_prefill_step", "xb_gemm_bf16",
)
TRACE_STAGES = 512
TRACE_STRIDE = 3 * TRACE_STAGES + 8
TRACE_BYTES = TRACE_STRIDE * 8 * 1024
STATIC_SCRATCH_BYTES = 4 << 20

vp = ctypes.c_void_p


class XbGeometry(ctypes.Structure):
    _fields_ = [
        ("family", ctypes.c_int32), ("num_layers", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32), ("vocab", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("rotary_dim", ctypes.c_int32),
        ("lin_key_heads", ctypes.c_int32), ("lin_value_heads", ctypes.c_int32),
        ("lin_head_dim", ctypes.c_int32), ("conv_width", ctypes.c_int32),
        ("capacity", ctypes.c_int32), ("state_rows", ctypes.c_int32),
        ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("rope_inv_freq", ctypes.POINTER(ctypes.c_float)),
        ("layer_kind", ctypes.c_int32 * MAX_LAYERS),
    ]


_LAYER_WEIGHT_FIELDS = (
    "input_norm", "post_norm", "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm",
    "in_qkv", "in_z", "in_b", "in_a", "conv_w", "a_log", "dt_bias", "gnorm", "out_proj",
    "gate", "up", "down",
)


class XbLayerWeights(ctypes.Structure):
    _fields_ = [(name, vp) for name in _LAYER_WEIGHT_FIELDS]


class XbModelWeights(ctypes.Structure):
    _fields_ = [
        ("embed", vp), ("final_norm", vp), ("lm_head", vp),
        ("layers", XbLayerWeights * MAX_LAYERS),
    ]


class XbLayerState(ctypes.Structure):
    _fields_ = [
        ("k_cache", vp), ("v_cache", vp), ("conv_in", vp), ("rec_in", vp),
        ("conv_out", vp), ("rec_out", vp),
    ]


class XbStepArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("input_ids", vp), ("cache_position", vp),
        ("host_ids", ctypes.c_int64 * MAX_BATCH), ("host_positions", ctypes.c_int64 * MAX_BATCH),
        ("kv_lengths", ctypes.c_int32 * MAX_BATCH),
        ("query_lengths", ctypes.c_int32 * MAX_BATCH),
        ("layers", XbLayerState * MAX_LAYERS),
        ("logits", vp), ("next_tokens", vp),
    ]


class NativeError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


_lib = None


class XbAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("q", vp), ("k", vp), ("v", vp), ("out", vp), ("strides", ctypes.c_longlong * 9),
        ("batch", ctypes.c_int32), ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("q_tokens", ctypes.c_int32), ("capacity", ctypes.c_int32),
        ("cu_offsets", vp), ("count", ctypes.c_int32), ("length", ctypes.c_int32),
        ("scale", ctypes.c_float), ("blocks", vp), ("blocks_stride", ctypes.c_longlong),
    ]


class XbPrefillArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", ctypes.c_int32), ("input_ids", vp), ("start_position", ctypes.c_int64),
        ("layers", XbLayerState * MAX_LAYERS), ("logits", vp), ("next_token", vp),
    ]


def library_path():
    override = os.environ.get("XINFER_B200_LIBRARY")
    return Path(override).resolve() if override else LIBRARY_PATH


def load():
    """Load the C-ABI library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.is_file():
        raise FileNotFoundError(
            f"{path} is missing: build it with `python -m xinfer_b200.build` "
            "(there is no CPU fallback for the decode path)"
        )
    lib = ctypes.CDLL(str(path))
    i32, sz = ctypes.c_int32, ctypes.c_size_t
    sig = {
        "xb_model_create": (i32, [ctypes.POINTER(XbGeometry), ctypes.POINTER(XbModelWeights),
                                  ctypes.POINTER(vp)]),
        "xb_model_destroy": (i32, [vp]),
        "xb_decode_workspace_bytes": (i32, [vp, i32, ctypes.POINTER(sz)]),
        "xb_workspace_init": (i32, [vp, sz, vp]),
        "xb_decode_step": (i32, [vp, ctypes.POINTER(XbStepArgs), vp, sz, vp]),
        "xb_workspace_check": (i32, [vp, vp, ctypes.POINTER(i32)]),
        "xb_rope_inv_freq": (i32, [ctypes.c_float, i32, ctypes.POINTER(ctypes.c_float)]),
        "xb_prefix_attention": (i32, [ctypes.POINTER(XbAttentionArgs), vp]),
        "xb_prefill_workspace_bytes": (i32, [vp, i32, ctypes.POINTER(sz)]),
        "xb_prefill_step": (i32, [vp, ctypes.POINTER(XbPrefillArgs), vp, sz, vp]),
        "xb_gemm_bf16": (i32, [i32, i32, i32, vp, vp, vp, vp]),
        "xb_decode_step_static": (i32, [ctypes.POINTER(XbGeometry), ctypes.POINTER(XbModelWeights),
                                        ctypes.POINTER(XbStepArgs), vp, ctypes.POINTER(i32)]),
        "xb_debug_trace": (i32, [vp, sz]),
        "xb_debug_fault": (i32, [i32, ctypes.c_uint64]),
        "xb_last_error": (ctypes.c_char_p, []),
        "xb_abi_version": (i32, []),
    }
    for name, (restype, argtypes) in sig.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.xb_abi_version() != 1:
        raise RuntimeError("xinfer_b200 ABI version mismatch")
    _lib = lib
    return lib


def check(code):
    if code != XB_OK:
        message = (load().xb_last_error() or b"").decode(errors="replace")
        raise NativeError(code, f"xinfer_b200 error {code}: {message}")


def rope_inv_freq(theta, rotary_dim):
    out = (ctypes.c_float * (rotary_dim // 2))()
    check(load().xb_rope_inv_freq(ctypes.c_float(theta), rotary_dim, out))
    return list(out)
