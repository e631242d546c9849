"""ctypes binding of ``libcv3cuda.so`` (the C ABI declared in ``include/cv3cuda.h``).

The library is loaded from the package directory.  There is no fallback: if it
is missing, or no CUDA device is present, every operation raises.  Each call
checks the returned status and raises the exception type the reference raises
for the same condition (ValueError / IndexError), RuntimeError otherwise.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcv3cuda.so")

CV3_OK, CV3_ERR_VALUE, CV3_ERR_INDEX, CV3_ERR_CUDA, CV3_ERR_UNSUPPORTED = 0, 1, 2, 3, 4

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F = ctypes.c_float
D = ctypes.c_double
U64 = ctypes.c_uint64

# name -> argument types (restype is always int status unless listed in _RESTYPE)
SIGNATURES = {
    "cv3_abi_version": [],
    "cv3_launch_count": [],
    "cv3_device_info": [P, P, P],
    "cv3_device_alloc": [I64, P],
    "cv3_device_free": [P],
    "cv3_memcpy": [P, P, I64, I32, P],
    "cv3_memset": [P, I32, I64, P],
    "cv3_stream_synchronize": [P],
    "cv3_mem_get_info": [P, P],
    "cv3_q8_linear": [P, I64, I64, I64, P, P, I64, I64, P, P, P, I64, P],
    "cv3_f32_linear": [P, I64, I64, I64, P, I64, I64, P, P, P, I64, P],
    "cv3_q8_dequant": [P, P, I64, I64, I64, P, P],
    "cv3_q4_linear": [P, I64, I64, I64, P, P, I64, I64, P, P, P, I64, P],
    "cv3_q4_dequant": [P, P, I64, I64, I64, P, P],
    "cv3_unary": [I32, F, P, I64, P, P],
    "cv3_rms_norm": [P, P, I64, I64, F, P, P],
    "cv3_layer_norm": [P, P, P, I64, I64, F, P, P],
    "cv3_softmax": [P, I64, I64, I32, P, P],
    "cv3_snake": [P, P, I64, I64, I64, P, P],
    "cv3_embedding": [P, I32, P, I64, I64, I64, P, I64, P, I64, P, P],
    "cv3_conv1d": [P, I64, I64, I64, P, I64, I64, I64, I64, I64, I64, I64, P, P, I64, P],
    "cv3_attention": [P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64, P, I64, I64, I64,
                      I64, I64, I64, I64, I64, I64, F, I32, I64, I64, P],
    "cv3_stft": [P, I64, I64, I64, I64, P, P, I64, P],
    "cv3_istft": [P, I32, I64, I64, I64, I64, P, F, I64, P, P, I64, P],
    "cv3_istft_noalloc": [P, I32, I64, I64, I64, I64, P, F, I64, P, I64, P],
    "cv3_interpolate_nearest": [P, I64, I64, I64, P, P],
    "cv3_interpolate_linear": [P, I64, I64, P, P, P, I64, P, P],
    "cv3_torch_rand": [U64, I64, I64, P, P],
    "cv3_torch_randn": [U64, I64, I64, P, P, P],
    "cv3_torch_u32": [U64, I64, I64, P, P],
    "cv3_torch_rand64": [U64, I64, I64, P, P],
    "cv3_rope_qkv_append": [P, I64, I64, P, P, P, P, I64, I64, I64, P, P, P, I64, P],
    "cv3_decode_attention": [P, P, P, P, I64, I64, I64, I64, I64, F, P, P],
    "cv3_decode_rope_attention": [P, I64, P, P, P, P, P, P, I64, I64, I64, I64, I64, F, P, P],
    "cv3_swiglu": [P, I64, I64, P, P],
    "cv3_head_select": [P, I64, I64, I64, P, P, P, P, P, I64, P, P],
    "cv3_sample_select": [P, I64, I64, I64, P, P, I32, D, I64, I64, D, P, P, P, P, P, I64, P, P, P, P],
    "cv3_dit_input_cat": [P, P, P, P, I64, I64, I64, I64, P, P],
    "cv3_ln_modulate": [P, I64, I64, F, P, P, I64, I64, P, P],
    "cv3_gate_residual": [P, P, P, I64, I64, I64, I64, P],
    "cv3_partial_rope": [P, I64, I64, I64, I64, I64, P, P, P],
    "cv3_transpose": [P, I64, I64, I64, P, I32, P],
    "cv3_cfg_euler": [P, P, I64, I64, I64, D, F, P],
    "cv3_l2_normalize": [P, I64, I64, P, P],
    "cv3_f0_classifier": [P, I64, I64, I64, P, P, P, P],
    "cv3_nsf_source": [P, I64, I64, I64, I64, I64, D, D, D, P, P, P, P, P, P],
    "cv3_binary": [I32, P, P, F, I64, P, P],
    "cv3_reflect_left1": [P, I64, I64, P, P],
    "cv3_tc_gemm": [P, I64, P, I64, P, I64, I64, I64, I64, I32, P, P, I64, I64, P],
    "cv3_tc_gemm_status": [P],
    "cv3_tf32_lo": [P, I64, P, P],
    "cv3_tc_gemm_split": [P, I64, P, P, I64, P, I64, I64, I64, I64, I32, P, P, I64, I64, P],
    "cv3_tc_attention_status": [P],
    "cv3_conv_weight_tc": [P, I64, I64, I64, I64, P, P, P],
    "cv3_conv1d_tc": [P, I64, I64, I64, I64, I64, I64, P, P, I64, I64, I64, I64, I64, I64, I64, P, I32, F, P,
                      P, P, I64, I64, I64, I64, P],
    "cv3_tc_conv_status": [P],
    "cv3_conv_tc_set_window": [I32],
    "cv3_set_dependent_launch": [I32],
    "cv3_conv_tc_last_path": [P],
    "cv3_tc_gemm_q8": [P, I64, P, P, P, I64, I64, I64, I64, I32, P, P, I64, I64, P],
    "cv3_q8_gemm_prepare": [P, P, I64, I64, P, P, P],
    "cv3_tc_gemm_q8_status": [P],
    "cv3_tc_gemm_q8_planes": [P, P, I64, P, P, P, I64, I64, I64, I64, I32, P, P, I64, I64, P, P, I64, P],
    "cv3_q8_split_rows": [P, I64, I64, I64, P, P, I64, P],
    "cv3_ln_modulate_planes": [P, I64, I64, F, P, P, I64, I64, P, P, I64, P],
    "cv3_decode_steps": [P, P],
    "cv3_decode_sync_words": [I64, I64],
    "cv3_decode_status": [P],
    "cv3_q8_decode_gemv": [P, I64, I64, I64, P, P, I64, I64, P, P, P, F, I32, P, I64, I64, P, I64, P, P],
    "cv3_q8_decode_gemv_mma": [P, I64, I64, I64, P, P, I64, I64, P, P, P, F, I32, P, I64, I64, P, I64, P, P],
    "cv3_decode_gemv_status": [P],
    "cv3_decode_attention_status": [P],
}
_RESTYPE = {"cv3_last_error": ctypes.c_char_p, "cv3_launch_count": ctypes.c_ulonglong,
            "cv3_decode_sync_words": ctypes.c_int64}

_lib: Optional[ctypes.CDLL] = None


EPI_BIAS, EPI_GELU, EPI_GATED_RESIDUAL, EPI_RESIDUAL = 0, 1, 2, 3


def exported_names():
    return ["cv3_last_error"] + list(SIGNATURES)


def launch_count() -> int:
    """Kernels launched or graph-recorded by the library so far (``cv3_launch_count``)."""
    return int(load().cv3_launch_count())


_graph_books = {"captured": 0, "replayed": 0}


def note_capture(nodes: int) -> None:
    _graph_books["captured"] += nodes


def note_replay(nodes: int) -> None:
    _graph_books["replayed"] += nodes


def executed_launches() -> int:
    """Kernels of this library executed so far: direct launches plus the kernel
    nodes of every CUDA-graph replay (recording during capture is not execution)."""
    return launch_count() - _graph_books["captured"] + _graph_books["replayed"]


class DecodeParams(ctypes.Structure):
    """``cv3_decode_params`` (include/cv3cuda.h), field for field."""
    _fields_ = [
        ("layers", ctypes.c_void_p),
        ("n_layers", ctypes.c_int32), ("batch", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("eps", ctypes.c_float), ("scale", ctypes.c_float),
        ("cap", ctypes.c_int64),
        ("cos_table", ctypes.c_void_p), ("sin_table", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
        ("head_q", ctypes.c_void_p), ("head_s", ctypes.c_void_p),
        ("vocab", ctypes.c_int32), ("select", ctypes.c_int32),
        ("emb", ctypes.c_void_p), ("emb_scales", ctypes.c_void_p), ("emb_rows", ctypes.c_int32),
        ("h", ctypes.c_void_p), ("h1", ctypes.c_void_p), ("qkv", ctypes.c_void_p), ("attn_part", ctypes.c_void_p),
        ("attn", ctypes.c_void_p), ("part", ctypes.c_void_p), ("part_floats", ctypes.c_int64), ("act", ctypes.c_void_p),
        ("logits", ctypes.c_void_p), ("logp", ctypes.c_void_p),
        ("pos", ctypes.c_void_p), ("lens", ctypes.c_void_p), ("next_ids", ctypes.c_void_p),
        ("history", ctypes.c_void_p), ("hist_stride", ctypes.c_int64),
        ("step", ctypes.c_void_p), ("sync", ctypes.c_void_p), ("sync_words", ctypes.c_int64),
        ("steps", ctypes.c_int32), ("trace_step", ctypes.c_int32), ("trace", ctypes.c_void_p),
    ]


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once) and attach signatures; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libcv3cuda.so not found at {path}; build it with "
            f"`python cosyvoice3-cpu_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    lib.cv3_last_error.restype = ctypes.c_char_p
    lib.cv3_last_error.argtypes = []
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    _lib = lib
    return lib


class CudaOpError(RuntimeError):
    pass


def check(status: int, name: str) -> None:
    if status == CV3_OK:
        return
    msg = (_lib.cv3_last_error() or b"").decode("utf-8", "replace")
    if status == CV3_ERR_VALUE:
        raise ValueError(msg)
    if status == CV3_ERR_INDEX:
        raise IndexError(msg)
    raise CudaOpError(f"{name}: {msg}")


def call(name: str, *args) -> None:
    lib = load()
    check(getattr(lib, name)(*args), name)
