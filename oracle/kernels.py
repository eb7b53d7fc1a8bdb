"""ctypes wrappers over the oracle's C restatement (``oracle/kernels.c``) and,
when built, the reference's own ``lut2_gather.c`` (``oracle/_ref``).

Test infrastructure: see ``oracle/__init__.py``.  Both libraries are CPU code;
``impl="oracle"`` calls the restatement, ``impl="reference"`` calls the
reference's exported C kernels with the argument conventions of its Python
dispatch (``rwkv_ssd/runtime/lut_gemm_fused.py:467-724``, ``:1336-1373``,
``:1562-1629``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "liblut2_gather.so"

_F = ctypes.POINTER(ctypes.c_float)
_U8 = ctypes.POINTER(ctypes.c_uint8)
_libs: dict[str, ctypes.CDLL] = {}


def build(quiet: bool = True) -> None:
    """Run ``oracle/Makefile`` (the oracle C library, plus ``_ref`` when the
    reference sources are present)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def lib(impl: str = "oracle") -> ctypes.CDLL:
    if impl in _libs:
        return _libs[impl]
    path = ORACLE_SO if impl == "oracle" else REF_SO
    if not path.is_file():
        build()
    if not path.is_file():
        raise FileNotFoundError(f"{impl} CPU library not built: {path}")
    h = ctypes.CDLL(str(path))
    _libs[impl] = h
    return h


def host_threads() -> int:
    """Threads a CPU run may use: the physical cores of the host, bounded by
    this process's CPU affinity."""
    try:
        avail = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        avail = os.cpu_count() or 1
    try:
        import psutil

        phys = psutil.cpu_count(logical=False) or avail
    except Exception:  # noqa: BLE001
        phys = avail
    return max(1, min(avail, phys))


def set_threads(n: int, impl: str = "reference") -> int:
    """Set the OpenMP thread count of a CPU library explicitly (an inherited
    ``OMP_NUM_THREADS``, e.g. torchrun's 1, would otherwise win) and return it.
    ``omp_set_num_threads`` is looked up through the library's handle, so it is
    the OpenMP runtime that library actually links."""
    n = max(1, int(n))
    os.environ["OMP_NUM_THREADS"] = str(n)
    h = lib(impl)
    try:
        h.omp_set_num_threads(ctypes.c_int(n))
    except AttributeError:
        pass
    try:
        return int(h.omp_get_max_threads())
    except AttributeError:
        return n


def ref_available() -> bool:
    if not REF_SO.is_file():
        try:
            build()
        except Exception:
            return False
    return REF_SO.is_file()


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _bp(b: np.ndarray):
    return b.ctypes.data_as(_U8)


def _blob(b) -> np.ndarray:
    return np.frombuffer(bytes(b) if not isinstance(b, np.ndarray) else b, dtype=np.uint8)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).reshape(-1)


def sg8_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """``y = W @ x`` for an SG8 blob of W ``[out_f, in_f]``."""
    b, xv = _blob(blob), _f32(x)
    y = np.empty(out_f, dtype=np.float32)
    if impl == "oracle":
        lib().oracle_sg8_gemv(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    else:
        lib(impl).scale_u8_grouped_gemv_f32_export(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    return y


def lut2_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """``y = W @ x`` for a grouped LUT2 blob (kinds 3..7)."""
    b, xv = _blob(blob), _f32(x)
    y = np.empty(out_f, dtype=np.float32)
    if impl == "oracle":
        lib().oracle_lut2_grouped_gemv(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    else:
        lib(impl).trinity_grouped_lut2_gemv_f32_export(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    return y


def packed_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """Dispatch on the blob magic like ``lut2_gemv`` (``lut_gemm_fused.py:1095-1192``)."""
    magic = bytes(blob[:4])
    if magic == b"SG8\x01":
        return sg8_gemv(blob, x, out_f, in_f, impl)
    if magic[:3] == b"TR2" and magic[3] in (3, 4, 5, 6, 7):
        return lut2_gemv(blob, x, out_f, in_f, impl)
    if magic == b"TR2\x01":
        return lut2_tensor_gemv(blob, x, out_f, in_f, impl)
    raise ValueError(f"unsupported packed blob magic {magic!r}")


def sg8_transposed_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """``y = x @ W`` for a row-major SG8 blob of W ``[in_f, out_f]``."""
    b, xv = _blob(blob), _f32(x)
    y = np.empty(out_f, dtype=np.float32)
    fn = (lib().oracle_sg8_transposed_gemv if impl == "oracle"
          else lib(impl).scale_u8_grouped_transposed_gemv_f32_export)
    fn(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    return y


def sg8_tmix_adapters(blobs, xs, a0, C: int, ranks, impl: str = "oracle"):
    """Fused TMix adapters: blobs ``w1,w2,a1,a2,g1,g2[,v1,v2]``, xs ``xw,xa,xg[,xv]``.

    Returns ``(w, a, g, v_or_None)``.
    """
    has_v = len(blobs) == 8
    keep_b = [_blob(b) for b in blobs] + [np.zeros(1, np.uint8)] * (8 - len(blobs))
    keep_x = [_f32(x) for x in xs] + [np.zeros(1, np.float32)] * (4 - len(xs))
    bp = (_U8 * 8)(*[_bp(b) for b in keep_b])
    xp = (_F * 4)(*[_fp(x) for x in keep_x])
    rk = (ctypes.c_int * 4)(*[int(r) for r in (list(ranks) + [0] * 4)[:4]])
    a0v = _f32(a0)
    w, a, g = (np.empty(C, np.float32) for _ in range(3))
    v = np.empty(C, np.float32) if has_v else np.zeros(1, np.float32)
    fn = (lib().oracle_sg8_tmix_adapters if impl == "oracle"
          else lib(impl).scale_u8_grouped_transposed_tmix_fused_f32_export)
    fn(_fp(w), _fp(a), _fp(g), _fp(v), bp, xp, _fp(a0v), int(C), rk, int(has_v))
    return w, a, g, (v if has_v else None)


def sg8_cmix(key_blob, value_blob, x, ko: int, ki: int, vo: int, vi: int,
             impl: str = "oracle") -> np.ndarray:
    """``y = Wv @ relu(Wk @ x)^2`` for SG8 blobs."""
    kb, vb, xv = _blob(key_blob), _blob(value_blob), _f32(x)
    y = np.empty(vo, dtype=np.float32)
    fn = lib().oracle_sg8_cmix if impl == "oracle" else lib(impl).scale_u8_grouped_cmix_gemv_f32_export
    fn(_fp(y), _bp(kb), _bp(vb), _fp(xv), int(ko), int(ki), int(vo), int(vi))
    return y


def sg8_tmix_qkv(blobs, xs, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """Three SG8 GEMVs with distinct inputs; returns ``y[3, out_f]``."""
    kb = [_blob(b) for b in blobs]
    kx = [_f32(x) for x in xs]
    y = np.empty((3, out_f), dtype=np.float32)
    bp = (_U8 * 3)(*[_bp(b) for b in kb])
    xp = (_F * 3)(*[_fp(x) for x in kx])
    if impl == "oracle":
        lib().oracle_sg8_tmix_qkv(_fp(y), bp, xp, int(out_f), int(in_f), 3)
    else:
        lib(impl).scale_u8_grouped_tmix_qkv_gemv_f32_export(_fp(y), bp, xp, int(out_f), int(in_f))
    return y


def lut2_tensor_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """``y = W @ x`` for a per-tensor LUT2 blob (``TR2\\x01``), the row walk of
    ``lut2_gemv_f32`` (K3)."""
    b, xv = _blob(blob), _f32(x)
    y = np.empty(out_f, dtype=np.float32)
    if impl == "oracle":
        lib().oracle_lut2_tensor_gemv(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    else:
        cb = np.frombuffer(b.tobytes(), dtype=np.float32, offset=4, count=4).copy()
        pk = np.ascontiguousarray(b[20:])
        lib(impl).lut2_gemv_f32_export(_fp(y), _fp(cb), _bp(pk), _fp(xv), int(out_f), int(in_f))
    return y


def sg8_i8_gemv(blob, x, out_f: int, in_f: int, impl: str = "oracle") -> np.ndarray:
    """Activation-INT8 SG8 GEMV (K7)."""
    b, xv = _blob(blob), _f32(x)
    y = np.empty(out_f, dtype=np.float32)
    fn = lib().oracle_sg8_i8_gemv if impl == "oracle" else lib(impl).scale_u8_grouped_i8_gemv_f32_export
    fn(_fp(y), _bp(b), _fp(xv), int(out_f), int(in_f))
    return y
