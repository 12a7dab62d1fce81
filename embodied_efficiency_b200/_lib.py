"""ctypes binding of ``lib/libee_b200.so`` (declared in ``include/ee_b200.h``).

The shared library is the only compute path: every entry point here raises
``RuntimeError`` when the library is missing or a call returns an error code.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

c_void_p, c_int32, c_int64, c_float, c_size_t = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                  ctypes.c_float, ctypes.c_size_t)

# status codes / enums (ee_b200.h)
EE_OK = 0
EE_ERR_TIMEOUT = 7
EE_BF16, EE_F16, EE_F32 = 0, 1, 2
EE_W_DENSE, EE_W_INT8, EE_W_INT4, EE_W_UINT4Z = 0, 1, 2, 3
EE_EPI_BIAS, EE_EPI_GELU, EE_EPI_RESIDUAL = 1, 2, 4
EE_MODE_EULER, EE_MODE_VELOCITY = 0, 1
EE_NORM_LAYER, EE_NORM_RMS = 0, 1


class Linear(ctypes.Structure):
    _fields_ = [("weight", c_void_p), ("scales", c_void_p), ("zeros", c_void_p), ("bias", c_void_p),
                ("n", c_int32), ("k", c_int32), ("wkind", c_int32), ("group", c_int32),
                ("scale_dtype", c_int32), ("reserved", c_int32)]


class Norm(ctypes.Structure):
    _fields_ = [("weight", c_void_p), ("bias", c_void_p)]


class Block(ctypes.Structure):
    _fields_ = [("n1", Norm), ("nx", Norm), ("n2", Norm),
                ("qkv", Linear), ("proj", Linear), ("q_c", Linear), ("out_c", Linear),
                ("mlp0", Linear), ("mlp2", Linear), ("kv", c_void_p)]


class Expert(ctypes.Structure):
    _fields_ = [("d_model", c_int32), ("n_layers", c_int32), ("n_heads", c_int32),
                ("horizon", c_int32), ("action_dim", c_int32), ("prefix_len", c_int32),
                ("hidden", c_int32), ("batch", c_int32),
                ("act_dtype", c_int32), ("norm_kind", c_int32), ("self_attn", c_int32),
                ("reserved", c_int32), ("eps", c_float), ("reserved_f", c_float),
                ("freqs", c_void_p), ("in_proj", Linear), ("t_proj", Linear), ("out_proj", Linear),
                ("out_norm", Norm), ("blocks", c_void_p), ("kv_maps", c_void_p)]


# name -> (restype, argtypes); every symbol include/ee_b200.h declares
SIGNATURES = {
    "ee_strerror": (ctypes.c_char_p, [c_int32]),
    "ee_version": (c_int32, []),
    "ee_struct_size": (c_size_t, [c_int32]),
    "ee_pack_int4": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "ee_unpack_int4": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "ee_wq_gemm": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                             c_void_p]),
    "ee_check_expert": (c_int32, [ctypes.POINTER(Expert), ctypes.POINTER(Block), c_int32, c_int32]),
    "ee_encode_kv_maps": (c_int32, [ctypes.POINTER(Expert), ctypes.POINTER(Block), c_void_p, c_size_t,
                                    c_void_p]),
    "ee_flow_sample_workspace_bytes": (c_size_t, [ctypes.POINTER(Expert), c_int32]),
    "ee_flow_sample": (c_int32, [ctypes.POINTER(Expert), c_void_p, c_void_p, c_void_p, c_int32,
                                 c_int32, c_void_p, c_size_t, c_void_p]),
    "ee_read_status": (c_int32, [c_void_p, ctypes.POINTER(c_int32), c_void_p]),
    "ee_wq_gemm_status": (c_int32, [ctypes.POINTER(c_int32), c_int32]),
    "ee_dequant_weight": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                                    c_int32, c_int32, c_void_p]),
    "ee_layer_norm": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                c_float, c_int32, c_void_p]),
    "ee_attention": (c_int32, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                               c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, c_int64, c_int32, c_void_p]),
    "ee_time_embed": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    "ee_expert_head": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
                                 c_int64, c_int64, c_int32, c_void_p]),
    "ee_euler_step": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_float, c_int32, c_void_p]),
    "ee_flow_sample_traced": (c_int32, [ctypes.POINTER(Expert), c_void_p, c_void_p, c_void_p, c_int32,
                                        c_int32, c_void_p, c_size_t, c_void_p, c_void_p]),
    "ee_flow_sample_phases": (c_int32, [ctypes.POINTER(Expert), c_int32]),
    "ee_flow_sample_geometry": (c_int32, [ctypes.POINTER(Expert), ctypes.POINTER(c_int32),
                                          ctypes.POINTER(c_int32), ctypes.POINTER(c_size_t)]),
    "ee_barrier_selftest": (c_int32, [c_void_p, ctypes.c_uint64, c_void_p]),
    "ee_flow_sample_noalloc": (c_int32, [ctypes.POINTER(Expert), c_void_p, c_void_p, c_void_p, c_int32,
                                         c_int32, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.LIB


def load():
    """Load the library (no build). Raises RuntimeError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(f"{path} is missing: build it with "
                                   "`python -m embodied_efficiency_b200.build`")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().ee_strerror(int(code)).decode()


def check(rc: int, what: str):
    if rc != EE_OK:
        raise RuntimeError(f"{what} failed: {strerror(rc)} (code {rc})")


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def act_code(dtype) -> int:
    if dtype == torch.bfloat16:
        return EE_BF16
    if dtype == torch.float16:
        return EE_F16
    raise TypeError(f"activation dtype must be bfloat16 or float16, got {dtype}")


def scale_code(dtype) -> int:
    if dtype == torch.float32:
        return EE_F32
    if dtype == torch.float16:
        return EE_F16
    raise TypeError(f"scales must be float32 or float16, got {dtype}")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("embodied_efficiency_b200 kernels need CUDA tensors "
                               f"(got a tensor on {t.device}); there is no CPU path")


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()
