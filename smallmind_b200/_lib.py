"""ctypes binding of libsmallmind_cuda.so (the C-ABI declared in include/smallmind_cuda.h).

The shared library is built in-tree by ``smallmind_b200/csrc/Makefile``.  There
is no fallback: if the library is missing or cannot be loaded, importing this
module raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsmallmind_cuda.so")

SM_OK = 0
ERRORS = {-1: "INVALID_ARG", -2: "SHAPE", -3: "CUDA", -4: "OOM", -5: "UNSUPPORTED", -6: "STATE", -7: "TIMEOUT",
          -8: "NCCL"}
PTR_HOST, PTR_DEVICE = 0, 1
LAYOUT_INTENDED, LAYOUT_REFERENCE = 0, 1

(ROLE_ATTN_NORM, ROLE_WQ, ROLE_WK, ROLE_WV, ROLE_WO, ROLE_FFN_NORM, ROLE_W_GATE, ROLE_W_UP, ROLE_W_DOWN,
 ROLE_TOKEN_EMBD, ROLE_OUT_NORM, ROLE_OUTPUT) = range(12)


class ModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn_hidden", C.c_int), ("max_context", C.c_int),
        ("norm_eps", C.c_float), ("rope_theta", C.c_float),
    ]


class SamplingParams(C.Structure):
    """sm_sampling_params (include/smallmind_cuda.h)."""
    _fields_ = [("temperature", C.c_double), ("top_k", C.c_int), ("top_p", C.c_double), ("min_p", C.c_double),
                ("repetition_penalty", C.c_float), ("presence_penalty", C.c_float),
                ("frequency_penalty", C.c_float), ("repetition_window", C.c_int)]


SAMPLE_MAX_VOCAB = 53248


# name -> (restype, argtypes); every symbol declared in include/smallmind_cuda.h
vp, i, i64, f, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
PP = C.POINTER(C.c_void_p)
SIGNATURES = {
    "sm_version": (i, []),
    "sm_last_error": (i, [C.c_char_p, sz]),
    "sm_device_count": (i, [C.POINTER(C.c_int)]),
    "sm_ctx_create": (i, [i, PP]),
    "sm_ctx_destroy": (i, [vp]),
    "sm_ctx_set_stream": (i, [vp, vp]),
    "sm_stream_sync": (i, [vp]),
    "sm_ctx_device_status": (i, [vp]),
    "sm_ctx_launch_count": (i, [vp, C.POINTER(C.c_int64)]),
    "sm_sample": (i, [vp, vp, i, i, C.POINTER(SamplingParams), vp, vp, i, vp, vp, vp, i]),
    "sm_weight_upload": (i, [vp, i, i, i, i, vp, sz, vp, sz, i, PP]),
    "sm_weight_upload_device": (i, [vp, i, i, i, i, vp, sz, vp, sz, i, PP]),
    "sm_weight_destroy": (i, [vp]),
    "sm_weight_info": (i, [vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "sm_weight_nbytes": (i, [vp, C.POINTER(C.c_size_t)]),
    "sm_matmul": (i, [vp, vp, vp, i, i, i, i]),
    "sm_dequant": (i, [vp, vp, i]),
    "sm_quantize": (i, [vp, i, vp, i64, i, vp, vp]),
    "sm_op_rmsnorm": (i, [vp, vp, vp, vp, i, i, f, i]),
    "sm_op_rope": (i, [vp, vp, i, i, i, vp, f, i, i]),
    "sm_op_silu_mul": (i, [vp, vp, vp, vp, i, i]),
    "sm_attention": (i, [vp, vp, vp, vp, vp, i, i, i, i, i, i]),
    "sm_attention_decode": (i, [vp, vp, vp, vp, vp, vp, i, i, i, i, i]),
    "sm_attention_decode_noalloc": (i, [vp, vp, vp, vp, vp, vp, i, i, i, i, i]),
    "sm_model_create": (i, [vp, C.POINTER(ModelConfig), PP]),
    "sm_model_set_weight": (i, [vp, i, i, vp]),
    "sm_model_set_vector": (i, [vp, i, i, vp, sz]),
    "sm_model_finalize": (i, [vp]),
    "sm_model_destroy": (i, [vp]),
    "sm_model_nbytes": (i, [vp, C.POINTER(C.c_size_t)]),
    "sm_tp_unique_id": (i, [vp, sz]),
    "sm_tp_init": (i, [vp, i, i, vp, sz]),
    "sm_tp_allreduce": (i, [vp, vp, sz]),
    "sm_model_set_tp": (i, [vp, i]),
    "sm_kv_create": (i, [vp, i, i, PP]),
    "sm_kv_destroy": (i, [vp]),
    "sm_kv_reset": (i, [vp, i]),
    "sm_kv_length": (i, [vp, i, C.POINTER(C.c_int)]),
    "sm_kv_truncate": (i, [vp, i, i]),
    "sm_prefill_batch": (i, [vp, vp, vp, vp, vp, i, vp, vp]),
    "sm_kv_slide": (i, [vp, i, i]),
    "sm_kv_read": (i, [vp, i, i, i, i, vp, vp]),
    "sm_prefill": (i, [vp, vp, i, vp, i, vp, vp]),
    "sm_decode": (i, [vp, vp, vp, vp, i, vp, vp, i]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"SmallMind CUDA library not built: {LIB_PATH} (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class SmallMindCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class ShapeError(SmallMindCudaError, ValueError):
    """Shape / length mismatch — the reference throws ArgumentException."""


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().sm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "") -> int:
    if rc < 0:
        msg = last_error()
        if rc in (-1, -2):
            raise ShapeError(rc, f"{what}: {msg}")
        raise SmallMindCudaError(rc, f"{what}: {msg}")
    return rc
