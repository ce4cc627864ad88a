"""ctypes binding of libnq8.so (the C ABI declared in include/nq8.h).

The shared library is built in-tree (``nspeech_b200/_lib/libnq8.so``) by
``make -C nspeech_b200/csrc`` or ``__graft_entry__.build()``.  Loading fails
loudly when it is missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libnq8.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "nq8.h")

# status codes
NQ_OK = 0
NQ_ERR_ARG = -1
NQ_ERR_SHAPE = -2
NQ_ERR_ALIGN = -3
NQ_ERR_DTYPE = -4
NQ_ERR_CUDA = -5
NQ_ERR_TIMEOUT = -6
NQ_ERR_FORMAT = -7
NQ_ERR_IO = -8
NQ_ERR_NOT_INIT = -9
NQ_ERR_UNSUPPORTED = -10
NQ_ERR_DEVICE = -11

NQ_F32 = 0
NQ_BF16 = 1

NQ_EPI_NONE = 0
NQ_EPI_SILU = 1
NQ_EPI_GELU_ERF = 2
NQ_EPI_GLU_SIGMOID = 3
NQ_EPI_GLU_SILU = 4
NQ_EPI_RELU = 5

NQ_PACK_DEFAULT = 0
NQ_PACK_GLU = 1
NQ_MODE_QTILED = 2

NQ_ATTENTION_TCGEN05 = 0
NQ_ATTENTION_MMA_SYNC = 1

NQ_CONV_AUTO = 0
NQ_CONV_IM2COL = 1

NQ_GEMV_AUTO = 0
NQ_GEMV_SPLIT = 1
NQ_GEMV_CLUSTER = 2


class NqError(RuntimeError):
    """A non-zero status from libnq8 (carries the code and the library message)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libnq8 error {code}: {msg}")
        self.code = code


class EncoderConfig(ctypes.Structure):
    """nq_encoder_config (mirrors FastConformerConfig, src/parakeet/fast_conformer.rs:31-45)."""

    _fields_ = [("feat_in", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("ff_mult", ctypes.c_int), ("n_layers", ctypes.c_int), ("conv_kernel", ctypes.c_int),
                ("sub_channels", ctypes.c_int), ("scale_input", ctypes.c_int)]


_lib = None
_lock = threading.Lock()
_inited: set[int] = set()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); every function declared in include/nq8.h.
SIGNATURES = {
    "nq_init": (_I, [_I]),
    "nq_version": (ctypes.c_char_p, []),
    "nq_weight_from_q8_0": (_I, [_P, _I64, _I64, _I, ctypes.POINTER(_P)]),
    "nq_weight_from_f32": (_I, [_P, _I64, _I64, _I, ctypes.POINTER(_P)]),
    "nq_weight_from_gguf": (_I, [ctypes.c_char_p, ctypes.c_char_p, _I, ctypes.POINTER(_P)]),
    "nq_gguf_tensor_info": (_I, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(_I), ctypes.POINTER(_I64),
                                 ctypes.POINTER(_I64)]),
    "nq_weights_fuse": (_I, [ctypes.POINTER(_P), _I, _I, ctypes.POINTER(_P)]),
    "nq_weight_to_q8_0": (_I, [_P, _P]),
    "nq_weight_shape": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I)]),
    "nq_weight_free": (None, [_P]),
    "nq_linear": (_I, [_P, _P, _I, _I64, _I64, _P, _I, _P, _I, _I64, _P]),
    "nq_matmul": (_I, [_P, _P, _I, _P, _I, _I64, _P]),
    "nq_matmul_bias": (_I, [_P, _P, _I, _P, _P, _I, _I64, _P]),
    "nq_matmul_bias_gelu": (_I, [_P, _P, _I, _P, _P, _I, _I64, _P]),
    "nq_gemv_splitk": (_I, [_P, _P, _I, _P, _P, _I, _P]),
    "nq_gemv_glu_splitk": (_I, [_P, _P, _I, _P, _P, _I, _P]),
    "nq_gemv_qkv_splitk": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _I, _P]),
    "nq_encoder_create": (_I, [_P, ctypes.POINTER(_P)]),
    "nq_encoder_set_tensor": (_I, [_P, ctypes.c_char_p, _I, _P, ctypes.POINTER(_I64), _I]),
    "nq_encoder_load_gguf": (_I, [_P, ctypes.c_char_p]),
    "nq_encoder_finalize": (_I, [_P]),
    "nq_encoder_out_frames": (_I, [_I]),
    "nq_encoder_forward": (_I, [_P, _P, ctypes.POINTER(ctypes.c_int32), _I, _I, _P, ctypes.POINTER(ctypes.c_int32), _P]),
    "nq_encoder_forward_host": (_I, [_P, _P, ctypes.POINTER(ctypes.c_int32), _I, _I, _P,
                                     ctypes.POINTER(ctypes.c_int32), _P]),
    "nq_encoder_forward_host_async": (_I, [_P, _P, ctypes.POINTER(ctypes.c_int32), _I, _I, _P,
                                           ctypes.POINTER(ctypes.c_int32), _P]),
    "nq_encoder_wait": (_I, [_P]),
    "nq_encoder_launch_count": (_I, [_P, _I, _I]),
    "nq_encoder_free": (None, [_P]),
    "nq_profile_enable": (_I, [_I]),
    "nq_profile_read": (_I, [_I, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_double),
                             ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), _I]),
    "nq_last_error": (_I, [ctypes.c_char_p, _I]),
    "nq_status": (_I, [_P, ctypes.POINTER(_I)]),
    "nq_gemv_noalloc": (_I, [_P, _P, _I, _I64, _I64, _P, _I, _P, _I, _I64, _P]),
    "nq_conv1d_out_len": (_I64, [_I64, _I, _I, _I, _I]),
    "nq_conv1d": (_I, [_P, _P, _I, _I64, _I64, _I64, _I, _I, _I, _I, ctypes.c_float, _P, _I, _P, _I, _I64, _P]),
    "nq_conv_transpose1d_out_len": (_I64, [_I64, _I, _I, _I, _I]),
    "nq_conv_transpose1d_weight": (_I, [_P, _I64, _I64, _I, ctypes.POINTER(_P)]),
    "nq_conv_transpose1d": (_I, [_P, _P, _I, _I64, _I64, _I64, _I, _I, _I, _I, ctypes.c_float, _P, _I, _P, _I, _I64,
                                 _P]),
    "nq_gemv_resadd_ln": (_I, [_P, _P, _I, _I64, _I64, _P, _P, _P, _I64, _P, _P, ctypes.c_float, _P, _I, _I64, _P]),
    "nq_weight_keep_bf16": (_I, [_P, _I]),
    "nq_launch_counter": (_I, [ctypes.POINTER(_I64), _I]),
    "nq_set_gemm_path": (_I, [_I]),
    "nq_set_gemm_unit_tokens": (_I, [_I]),
    "nq_set_gemm_tail_split": (_I, [_I]),
    "nq_set_attention_kernel": (_I, [_I]),
    "nq_set_conv_path": (_I, [_I]),
    "nq_set_gemv_path": (_I, [_I]),
    "nq_chain_create": (_I, [ctypes.POINTER(_P)]),
    "nq_chain_linear": (_I, [_P, _P, _P, _P, _I, _P, _I]),
    "nq_chain_gemv_resadd_ln": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_float, _P]),
    "nq_chain_steps": (_I, [_P]),
    "nq_chain_run": (_I, [_P, _P]),
    "nq_chain_free": (None, [_P]),
    "nq_set_wait_limit": (_I, [_I64]),
    "nq_debug_wait_timeout": (_I, [_P]),
}


def load() -> ctypes.CDLL:
    """Load libnq8.so and bind every exported symbol (no CUDA work)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `make -C nspeech_b200/csrc` "
                    "(there is no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().nq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != NQ_OK:
        raise NqError(rc, last_error())


def init(device: int = 0) -> None:
    """nq_init for `device` on the calling thread (idempotent)."""
    L = load()
    check(L.nq_init(device))
    _inited.add(device)


def status(stream_ptr: int = 0) -> int:
    """Synchronize the stream and return the device status bits (0 = clean)."""
    bits = ctypes.c_int(0)
    rc = load().nq_status(_P(stream_ptr), ctypes.byref(bits))
    if rc not in (NQ_OK, NQ_ERR_TIMEOUT):
        check(rc)
    return bits.value


NQ_KCLASS_GEMM = 0
NQ_KCLASS_GEMV = 1
NQ_KCLASS_DEQUANT = 2
NQ_KCLASS_REDUCE = 3
NQ_KCLASS_ATTENTION = 4
NQ_KCLASS_NORM = 5
NQ_GEMM_AUTO = 0
NQ_GEMM_FUSED = 1
NQ_GEMM_DEQUANT = 2


def launch_counter(reset: bool = False) -> int:
    """Kernels launched by libnq8 in this process (optionally zeroing the count)."""
    n = ctypes.c_int64()
    check(load().nq_launch_counter(ctypes.byref(n), 1 if reset else 0))
    return n.value


def profile_enable(on: bool) -> None:
    check(load().nq_profile_enable(1 if on else 0))


def profile_read(kclass: int, reset: bool = True) -> dict:
    """Per-kernel-class launch count, device ms, algorithmic FLOPs and bytes."""
    n = ctypes.c_int64()
    ms, fl, by = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    check(load().nq_profile_read(kclass, ctypes.byref(n), ctypes.byref(ms), ctypes.byref(fl), ctypes.byref(by),
                                 1 if reset else 0))
    out = {"launches": n.value, "ms": ms.value, "flops": fl.value, "bytes": by.value}
    if ms.value > 0:
        out["tflops"] = fl.value / ms.value / 1e9
        out["gbs"] = by.value / ms.value / 1e6
    return out
