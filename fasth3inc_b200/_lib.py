"""ctypes binding of libfh3cuda (include/fh3cuda.h).

Loads the in-tree fasth3inc_b200/libfh3cuda.so.  There is no fallback: if the
library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

Q4_K = 12
F32 = 0
# the other formats fh3_dequant expands (fh3's enum values, include/fh3/fh3.h:64-78)
F16, BF16, Q8_0, Q2_K, Q3_K, Q5_K, Q6_K = 1, 30, 8, 10, 11, 13, 14

FH3_OK = 0
FH3_ERR = -1
FH3_E_NOMEM = -7
FH3_E_INVALID = -8
FH3CUDA_E_CUDA = -20
FH3CUDA_E_TIMEOUT = -21
FH3CUDA_E_NODEV = -22

EPI_F32, EPI_BF16, EPI_SWIGLU, EPI_RESID = 0, 1, 2, 3
GEMM_WEIGHTS_READY = 1

EXPORTED = [
    "fh3cuda_init", "fh3cuda_last_error", "fh3cuda_take_status", "fh3cuda_device_status",
    "fh3cuda_sm_count", "fh3cuda_row_bytes", "fh3cuda_dequant_dev", "fh3cuda_matmul_dev",
    "fh3cuda_matmul", "__wrap_fh3_matmul", "fh3cuda_register_weights", "fh3cuda_unregister_weights",
    "fh3cuda_upload_weights", "fh3cuda_release_weights", "fh3cuda_gemv_q4k_dev",
    "fh3cuda_gemm_q4k_dev", "fh3cuda_f32_to_bf16_dev", "fh3cuda_rmsnorm_modulate_dev",
    "fh3cuda_swiglu_dev", "fh3cuda_make_q4k_weights_dev", "fh3cuda_matmul_noalloc_dev",
    "fh3cuda_qk_norm_rope_dev", "fh3cuda_attention_dev", "fh3cuda_vsa_num_tiles", "fh3cuda_vsa_attention_dev",
    "fh3cuda_vsa_tiles_dev", "fh3cuda_attention_f32_dev", "fh3cuda_pack_open", "fh3cuda_pack_num_layers",
    "fh3cuda_pack_device_bytes", "fh3cuda_pack_layer", "fh3cuda_pack_close", "fh3cuda_adaln_open",
    "fh3cuda_adaln_dims", "fh3cuda_adaln_row", "fh3cuda_adaln_close", "fh3cuda_dit_prepare_text_dev",
    "fh3cuda_dit_forward_dev", "fh3cuda_gemm_launches", "fh3cuda_set_scratch_limit", "fh3cuda_alloc_stats",
    "fh3cuda_wait_selftest_dev", "fh3cuda_q4k_to_bf16_dev", "fh3cuda_gemm_bf16w_dev",
]


class Fh3CudaW(ctypes.Structure):
    """Same layout as fh3's Fh3W (include/fh3/fh3.h:82-87)."""
    _fields_ = [("type", ctypes.c_int), ("in_", ctypes.c_int64), ("out", ctypes.c_int64),
                ("data", ctypes.c_void_p)]


class Fh3CudaSeq(ctypes.Structure):
    """The fields of fh3's struct Fh3Seq (src/model/fh3_seq.h:31-38) that video sparse attention reads."""
    _fields_ = [("seq_len", ctypes.c_int32), ("num_text", ctypes.c_int32), ("num_audio", ctypes.c_int32),
                ("num_video", ctypes.c_int32), ("grid_t", ctypes.c_int32), ("grid_h", ctypes.c_int32),
                ("grid_w", ctypes.c_int32)]


class Fh3CudaLayerView(ctypes.Structure):
    """fh3's Fh3LayerView (include/fh3/fh3.h:90-100) with device pointers."""
    _fields_ = [(n, Fh3CudaW) for n in ("qkv", "gate_compress", "out", "fc1", "fc2", "norm1", "norm2", "q_norm",
                                        "k_norm")]


class Fh3CudaDitCfg(ctypes.Structure):
    """The fields of fh3's Fh3DitCfg (src/model/fh3_dit.h:19-39) the device forward uses (+ attn_bf16)."""
    _fields_ = [("attn", ctypes.c_int32), ("vsa_tile", ctypes.c_int32), ("vsa_sparsity", ctypes.c_float),
                ("hidden_size", ctypes.c_int32), ("num_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("num_layers", ctypes.c_int32), ("num_refiner_layers", ctypes.c_int32), ("ffn_dim", ctypes.c_int32),
                ("norm_eps", ctypes.c_float), ("qk_norm_eps", ctypes.c_float), ("final_norm_eps", ctypes.c_float),
                ("attn_bf16", ctypes.c_int32)]


class Fh3CudaRefinerBlock(ctypes.Structure):
    """fh3's Fh3RefinerBlock (src/model/fh3_dit.h:41-50) with device pointers."""
    _fields_ = [("norm1", ctypes.c_void_p), ("qkv", Fh3CudaW), ("q_norm", ctypes.c_void_p),
                ("k_norm", ctypes.c_void_p), ("out", Fh3CudaW), ("norm2", ctypes.c_void_p), ("fc1", Fh3CudaW),
                ("fc2", Fh3CudaW)]


class Fh3CudaDitGlobals(ctypes.Structure):
    """The global weights of fh3's Fh3Dit (src/model/fh3_dit.h:52-86) as device data."""
    _fields_ = [("video_patch_proj", Fh3CudaW), ("video_patch_proj_bias", ctypes.c_void_p),
                ("audio_patch_proj", Fh3CudaW), ("audio_patch_proj_bias", ctypes.c_void_p),
                ("condition_proj", Fh3CudaW), ("condition_proj_bias", ctypes.c_void_p),
                ("refiner", Fh3CudaRefinerBlock * 4), ("refiner_final_norm", ctypes.c_void_p),
                ("final_norm", ctypes.c_void_p), ("video_out", Fh3CudaW), ("video_out_bias", ctypes.c_void_p),
                ("audio_out", Fh3CudaW), ("audio_out_bias", ctypes.c_void_p)]


class Fh3CudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libfh3cuda.so (compiling it first if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise FileNotFoundError(f"{path} not built; run python -m fasth3inc_b200.build")
        _build.build()
    L = ctypes.CDLL(path)
    vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    Wp = ctypes.POINTER(Fh3CudaW)
    sig = {
        "fh3cuda_init": (c_int, [c_int]),
        "fh3cuda_last_error": (ctypes.c_char_p, []),
        "fh3cuda_take_status": (c_int, []),
        "fh3cuda_device_status": (c_int, [vp]),
        "fh3cuda_sm_count": (c_int, []),
        "fh3cuda_row_bytes": (ctypes.c_size_t, [c_int, i64]),
        "fh3cuda_dequant_dev": (c_int, [c_int, vp, vp, i64, i64, vp]),
        "fh3cuda_matmul_dev": (c_int, [Wp, vp, vp, c_int, vp, vp]),
        "fh3cuda_matmul_noalloc_dev": (c_int, [Wp, vp, vp, c_int, vp, vp]),
        "fh3cuda_matmul": (None, [Wp, vp, vp, c_int, vp]),
        "__wrap_fh3_matmul": (None, [Wp, vp, vp, c_int, vp]),
        "fh3cuda_register_weights": (c_int, [vp, ctypes.c_size_t, vp]),
        "fh3cuda_unregister_weights": (c_int, [vp]),
        "fh3cuda_upload_weights": (c_int, [vp, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "fh3cuda_release_weights": (c_int, [vp]),
        "fh3cuda_gemv_q4k_dev": (c_int, [Wp, vp, vp, c_int, vp, vp]),
        "fh3cuda_gemm_q4k_dev": (c_int, [Wp, vp, i64, vp, i64, i64, vp, vp, c_int, vp]),
        "fh3cuda_f32_to_bf16_dev": (c_int, [vp, vp, i64, vp]),
        "fh3cuda_rmsnorm_modulate_dev": (c_int, [vp, vp, vp, vp, vp, c_int, c_int, ctypes.c_float, vp]),
        "fh3cuda_swiglu_dev": (c_int, [vp, vp, c_int, c_int, vp]),
        "fh3cuda_qk_norm_rope_dev": (c_int, [vp, c_int, i64, vp, c_int, i64, vp, vp, vp, c_int, c_int, c_int,
                                              c_int, ctypes.c_float, vp]),
        "fh3cuda_attention_dev": (c_int, [vp, i64, vp, i64, vp, i64, vp, c_int, i64, c_int, c_int, c_int, vp]),
        "fh3cuda_make_q4k_weights_dev": (c_int, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, i64, i64,
                                                 vp, vp]),
        "fh3cuda_pack_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(vp)]),
        "fh3cuda_pack_num_layers": (c_int, [vp]),
        "fh3cuda_pack_device_bytes": (ctypes.c_uint64, [vp]),
        "fh3cuda_pack_layer": (c_int, [vp, c_int, ctypes.POINTER(Fh3CudaLayerView)]),
        "fh3cuda_pack_close": (None, [vp]),
        "fh3cuda_adaln_open": (c_int, [ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(vp)]),
        "fh3cuda_adaln_dims": (c_int, [vp] + [ctypes.POINTER(c_int)] * 4),
        "fh3cuda_adaln_row": (vp, [vp, c_int, c_int, c_int, c_int]),
        "fh3cuda_adaln_close": (None, [vp]),
        "fh3cuda_dit_prepare_text_dev": (c_int, [ctypes.POINTER(Fh3CudaDitCfg), ctypes.POINTER(Fh3CudaDitGlobals),
                                                 vp, c_int, vp, vp]),
        "fh3cuda_dit_forward_dev": (c_int, [ctypes.POINTER(Fh3CudaDitCfg), ctypes.POINTER(Fh3CudaDitGlobals), vp, vp,
                                            ctypes.POINTER(Fh3CudaSeq), vp, vp, c_int, vp, vp, vp, vp, vp, vp]),
        "fh3cuda_gemm_launches": (c_int, [i64]),
        "fh3cuda_set_scratch_limit": (None, [ctypes.c_uint64]),
        "fh3cuda_wait_selftest_dev": (c_int, [ctypes.c_uint64, vp]),
        "fh3cuda_q4k_to_bf16_dev": (c_int, [Wp, vp, vp]),
        "fh3cuda_gemm_bf16w_dev": (c_int, [vp, i64, i64, vp, i64, vp, i64, i64, vp, vp, c_int, c_int, vp]),
        "fh3cuda_alloc_stats": (None, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
        "fh3cuda_attention_f32_dev": (c_int, [vp, i64, vp, i64, vp, i64, vp, i64, c_int, c_int, c_int, vp]),
        "fh3cuda_vsa_num_tiles": (c_int, [ctypes.POINTER(Fh3CudaSeq), c_int, ctypes.POINTER(c_int),
                                          ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
        "fh3cuda_vsa_attention_dev": (c_int, [c_int, ctypes.c_float, ctypes.POINTER(Fh3CudaSeq), vp, i64, vp, i64,
                                              vp, i64, c_int, vp, i64, vp, c_int, i64, c_int, c_int, vp]),
        "fh3cuda_vsa_tiles_dev": (c_int, [c_int, ctypes.c_float, ctypes.POINTER(Fh3CudaSeq), vp, i64, vp, i64,
                                          c_int, c_int, c_int, vp, vp, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return load().fh3cuda_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != FH3_OK:
        raise Fh3CudaError(rc, last_error())


def alloc_stats() -> tuple[int, int]:
    """(cudaMalloc calls the library has made, scratch bytes it holds now)."""
    a, b = ctypes.c_uint64(0), ctypes.c_uint64(0)
    load().fh3cuda_alloc_stats(ctypes.byref(a), ctypes.byref(b))
    return int(a.value), int(b.value)


def set_scratch_limit(nbytes: int) -> None:
    """Budget for the library's scratch over all devices (0 = unlimited)."""
    load().fh3cuda_set_scratch_limit(int(nbytes))
