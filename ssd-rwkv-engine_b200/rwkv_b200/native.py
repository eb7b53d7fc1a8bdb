"""ctypes loader for the sm_100a library ``_lib/librwkvb200.so``.

Mirrors the reference's ``rwkv_ssd/native/lut2_gather_loader.py`` (``lib()``,
``native_lib_path()``, ``build_native()``), with one deliberate difference:
there is no soft failure.  The reference logs and returns ``None`` so that
Python can fall back to Numba/NumPy (``lut_gemm_fused.py:1123-1157``); this
library has no CPU fallback, so a missing or unloadable library raises.

The C declarations live in ``include/rwkv_b200.h``; the ctypes structures
below mirror them field for field.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

_LIB: ctypes.CDLL | None = None
_LOCK = threading.Lock()

RWKVB_OK = 0
RWKVB_EARG = 1
RWKVB_EALLOC = 2
RWKVB_ECUDA = 3
RWKVB_ETIMEOUT = 4
RWKVB_EUNSUPPORTED = 5
RWKVB_ESCRATCH = 6
CMIX_NOALLOC_MAX_FFN = 16384

KIND_SG8 = 1
KIND_LUT2_TENSOR = 33  # TR2\x01 (per-tensor LUT2)
LUT2_KINDS = (3, 4, 5, 6, 7)

# Engine flags (rwkvb_engine_create)
FLAG_NO_GRAPH = 0x1
FLAG_NO_PDL = 0x2
FLAG_LUT2_CUDA_CORES = 0x4  # batch engines with LUT2 packs: fp32 CUDA-core products
FLAG_NO_PERSISTENT = 0x4
FLAG_TRACE = 0x8
FLAG_EXPLICIT_PREFETCH = 0x100
FLAG_NO_L2_POLICY = 0x200
FLAG_RING_SLOTS_SHIFT = 12  # bits 12..15: persistent-kernel ring slots, 3..8 (0: default 3)
FLAG_FFN_ROW_ORDER = 0x10000  # persistent kernel: FFN value units in row order, fp32 accumulation


class RwkvbError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, status: int, what: str):
        self.status = status
        text = "unknown"
        try:
            text = lib().rwkvb_status_string(status).decode()
        except Exception:
            pass
        super().__init__(f"{what} failed: {text} (status {status})")


class Packed(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("bytes", ctypes.c_uint64), ("kind", ctypes.c_uint32),
                ("group_size", ctypes.c_uint32), ("rows", ctypes.c_int32), ("cols", ctypes.c_int32)]


_FP = ctypes.c_void_p  # device float*


class LayerDesc(ctypes.Structure):
    _fields_ = ([(n, Packed) for n in ("att_r", "att_k", "att_v", "att_o", "w1", "w2", "a1", "a2", "g1", "g2",
                                        "v1", "v2", "ffn_key", "ffn_value")]
                + [(n, _FP) for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "x_r", "x_w", "x_k", "x_v", "x_a", "x_g",
                                       "w0", "a0", "v0", "k_k", "k_a", "r_k", "lnx_w", "lnx_b", "ffn_x_k")])


class ModelDesc(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int32), ("n_embd", ctypes.c_int32), ("head_size", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("vocab", ctypes.c_int32), ("emb", Packed), ("head", Packed),
                ("ln0_w", _FP), ("ln0_b", _FP), ("ln_out_w", _FP), ("ln_out_b", _FP),
                ("layers", ctypes.POINTER(LayerDesc))]


# void (*)(int32 kind, void* send, void* recv, int64 bytes, void* stream, void* user)
COLLECTIVE_FN = ctypes.CFUNCTYPE(None, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                 ctypes.c_void_p, ctypes.c_void_p)
COLLECTIVE_ALLREDUCE_SUM_F32 = 0
COLLECTIVE_ALLGATHER = 1


class TPDesc(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("size", ctypes.c_int32), ("vocab_offset", ctypes.c_int32),
                ("collective", COLLECTIVE_FN), ("user", ctypes.c_void_p),
                ("peer", ctypes.POINTER(ctypes.c_void_p))]


class StageDesc(ctypes.Structure):
    _fields_ = [("n_slots", ctypes.c_int32), ("slot_of_layer", ctypes.POINTER(ctypes.c_int32)),
                ("host_src", ctypes.POINTER(ctypes.c_void_p)), ("slot_dev", ctypes.POINTER(ctypes.c_void_p)),
                ("layer_bytes", ctypes.c_uint64)]


def native_lib_path() -> Path | None:
    return _build.LIB if _build.LIB.is_file() else None


def build_native(*, verbose: bool = False) -> Path:
    return _build.build(verbose=verbose)


EXPORTS: dict[str, tuple[object, list]] = {}


def _declare(h: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    vp, i32, u32, u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64
    sig = {
        "rwkvb_version": (ctypes.c_int, []),
        "rwkvb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
        "rwkvb_packed_init": (ctypes.c_int, [P(Packed), ctypes.c_char_p, u64, vp, i32, i32]),
        "rwkvb_dequant_f32": (ctypes.c_int, [vp, P(Packed), vp]),
        "rwkvb_gemv_f32": (ctypes.c_int, [vp, P(Packed), vp, vp]),
        "rwkvb_transposed_gemv_f32": (ctypes.c_int, [vp, P(Packed), vp, vp]),
        "rwkvb_tmix_qkv_gemv_f32": (ctypes.c_int, [vp, P(P(Packed)), P(vp), vp]),
        "rwkvb_tmix_gemv_f32": (ctypes.c_int, [vp, P(P(Packed)), P(vp), i32, vp]),
        "rwkvb_gemv_sg8_i8_f32": (ctypes.c_int, [vp, P(Packed), vp, vp]),
        "rwkvb_tmix_qkv_i8_gemv_f32": (ctypes.c_int, [vp, P(P(Packed)), P(vp), vp]),
        "rwkvb_tmix_adapters_f32": (ctypes.c_int, [vp, vp, vp, vp, P(P(Packed)), P(vp), vp, ctypes.c_int, vp]),
        "rwkvb_cmix_gemv_f32": (ctypes.c_int, [vp, P(Packed), P(Packed), vp, vp]),
        "rwkvb_cmix_gemv_f32_noalloc": (ctypes.c_int, [vp, P(Packed), P(Packed), vp, vp]),
        "rwkvb_gemm_sg8_f32": (ctypes.c_int, [vp, P(Packed), vp, i32, vp, vp]),
        "rwkvb_wkv7_f32": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, vp]),
        "rwkvb_engine_create": (ctypes.c_int, [P(ModelDesc), u32, P(vp)]),
        "rwkvb_engine_destroy": (ctypes.c_int, [vp]),
        "rwkvb_engine_create_staged": (ctypes.c_int, [P(ModelDesc), P(StageDesc), u32, P(vp)]),
        "rwkvb_engine_buffers": (ctypes.c_int, [vp, P(vp), P(vp), P(vp), P(vp)]),
        "rwkvb_engine_reset": (ctypes.c_int, [vp, vp]),
        "rwkvb_engine_forward": (ctypes.c_int, [vp, P(i32), i32, vp]),
        "rwkvb_engine_decode_greedy": (ctypes.c_int, [vp, i32, i32, P(i32), vp]),
        "rwkvb_engine_decode_greedy_async": (ctypes.c_int, [vp, i32, i32, vp, vp]),
        "rwkvb_engine_launches_per_step": (ctypes.c_int, [vp, P(i32)]),
        "rwkvb_engine_trace": (ctypes.c_int, [vp, P(u64), i32, P(i32)]),
        "rwkvb_engine_host_ring": (ctypes.c_int, [vp, P(vp), P(vp), P(vp), P(i32)]),
        "rwkvb_engine_decode_stream": (ctypes.c_int, [vp, i32, i32, vp, vp]),
        "rwkvb_engine_check": (ctypes.c_int, [vp, vp]),
        "rwkvb_batch_create": (ctypes.c_int, [P(ModelDesc), i32, u32, P(vp)]),
        "rwkvb_batch_create_tp": (ctypes.c_int, [P(ModelDesc), i32, P(TPDesc), u32, P(vp)]),
        "rwkvb_batch_prepare": (ctypes.c_int, [vp, vp]),
        "rwkvb_batch_tp_exchange_bytes": (ctypes.c_int, [P(ModelDesc), i32, P(u64)]),
        "rwkvb_ipc_alloc": (ctypes.c_int, [u64, P(vp), ctypes.c_char_p]),
        "rwkvb_ipc_free": (ctypes.c_int, [vp]),
        "rwkvb_ipc_open": (ctypes.c_int, [ctypes.c_char_p, P(vp)]),
        "rwkvb_ipc_close": (ctypes.c_int, [vp]),
        "rwkvb_batch_destroy": (ctypes.c_int, [vp]),
        "rwkvb_batch_buffers": (ctypes.c_int, [vp, P(vp), P(vp), P(vp), P(vp)]),
        "rwkvb_batch_reset": (ctypes.c_int, [vp, vp]),
        "rwkvb_batch_forward": (ctypes.c_int, [vp, P(i32), vp]),
        "rwkvb_batch_prefill": (ctypes.c_int, [vp, P(i32), i32, vp]),
        "rwkvb_batch_decode_greedy": (ctypes.c_int, [vp, i32, P(i32), vp]),
        "rwkvb_batch_decode_greedy_async": (ctypes.c_int, [vp, i32, vp, vp]),
        "rwkvb_batch_launches_per_step": (ctypes.c_int, [vp, P(i32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(h, name)  # AttributeError if the build lacks a declared symbol
        fn.restype = res
        fn.argtypes = args
        EXPORTS[name] = (res, args)


def lib() -> ctypes.CDLL:
    """Load (building first if needed) and return the library.  Raises on failure."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.build()
            h = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
            _declare(h)
            if h.rwkvb_version() != 1:
                raise RuntimeError("librwkvb200 ABI version mismatch")
            _LIB = h
    return _LIB


def check(status: int, what: str) -> None:
    if status != RWKVB_OK:
        raise RwkvbError(status, what)
