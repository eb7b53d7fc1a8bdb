"""Device mirror of the reference's fused packed-GEMV dispatch.

Same function names, argument meaning and error behaviour as
``rwkv_ssd/runtime/lut_gemm_fused.py`` in the reference engine, computed by
the sm_100a library through its C ABI on CUDA tensors:

=====================================  ===========================================  =========================
function                               reference                                    C ABI
=====================================  ===========================================  =========================
``lut2_gemv``                          ``lut_gemm_fused.py:1095-1192``              ``rwkvb_gemv_f32``,
                                                                                    ``rwkvb_gemv_sg8_i8_f32``
``lut2_tmix_gemv_batched``             ``lut_gemm_fused.py:1724-1769``              ``rwkvb_tmix_gemv_f32``
``lut2_tmix_qkv_gemv_batched``         ``lut_gemm_fused.py:1771-1817``              ``rwkvb_tmix_qkv_gemv_f32``,
                                                                                    ``rwkvb_tmix_qkv_i8_gemv_f32``
``lut2_layer_gather``                  ``lut2_gather.c:135-171``                    ``rwkvb_dequant_f32``
``grouped_u8_transposed_gemv``         ``lut_gemm_fused.py:1195-1233``              ``rwkvb_transposed_gemv_f32``
``grouped_u8_transposed_tmix_fused``   ``lut_gemm_fused.py:704-724``                ``rwkvb_tmix_adapters_f32``
``grouped_u8_cmix_gemv``               ``lut_gemm_fused.py:1431-1495``              ``rwkvb_cmix_gemv_f32``
``decode_packed``                      ``pack_codec.py:126-144``,                   ``rwkvb_dequant_f32``
                                       ``trinity_codec.py:754-885``
=====================================  ===========================================  =========================

``weight_blob`` arguments accept either a ``residency.DevicePacked`` (already
resident in HBM — the normal engine path) or the raw wire bytes, which are
uploaded for the call.  Activations may be CPU or CUDA tensors; results are
fp32 CUDA tensors on the current device (the reference returns the input's
dtype/device; callers here live on the GPU).  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import native
from .residency import DevicePacked, WeightArena

SG8_MAGIC = b"SG8\x01"


def _dev() -> torch.device:
    return torch.device("cuda", torch.cuda.current_device())


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _resident(blob, rows: int, cols: int, keep: list) -> DevicePacked:
    if isinstance(blob, DevicePacked):
        if blob.shape != (rows, cols):
            raise ValueError(f"packed shape {blob.shape} != ({rows}, {cols})")
        return blob
    raw = bytes(blob)
    codec = "sg8" if raw[:4] == SG8_MAGIC else "lut2"
    arena = WeightArena([("w", raw, (int(rows), int(cols)), codec)], _dev())
    keep.append(arena)
    return arena["w"]


def _vec(x: torch.Tensor, n: int, what: str = "x") -> torch.Tensor:
    t = x.detach().reshape(-1).to(device=_dev(), dtype=torch.float32).contiguous()
    if t.numel() != n:
        raise ValueError(f"{what} size {t.numel()} != in_features {n}")
    return t


def _magic(blob) -> bytes:
    if isinstance(blob, DevicePacked):
        return SG8_MAGIC if blob.codec == "sg8" else b"TR2"
    return bytes(blob[:4])


def activation_int8_enabled(*, head: bool = False) -> bool:
    """Whether the opt-in activation-INT8 SG8 GEMV is on: the reference's
    switches ``RWKV_LUT_ACTIVATION_INT8`` / ``..._HEAD`` (lut_gemm_fused.py:54-66)."""
    name = "RWKV_LUT_ACTIVATION_INT8_HEAD" if head else "RWKV_LUT_ACTIVATION_INT8"
    return os.environ.get(name, "0").strip().lower() in ("1", "true", "yes", "on")


def lut2_gemv(weight_blob, x: torch.Tensor, *, out_features: int, in_features: int,
              activation_int8: bool | None = None) -> torch.Tensor:
    """``y = W @ x`` for an SG8, grouped-LUT2 or per-tensor LUT2 (``TR2\\x01``)
    ``W [out_features, in_features]``; SG8 with ``activation_int8`` (default:
    ``activation_int8_enabled()``) quantises x per group to int8 first."""
    if activation_int8 is None:
        activation_int8 = activation_int8_enabled()
    keep: list = []
    w = _resident(weight_blob, out_features, in_features, keep)
    xv = _vec(x, in_features)
    y = torch.empty(out_features, dtype=torch.float32, device=_dev())
    if activation_int8 and w.codec == "sg8":
        native.check(native.lib().rwkvb_gemv_sg8_i8_f32(y.data_ptr(), ctypes.byref(w.desc), xv.data_ptr(),
                                                        _stream()), "rwkvb_gemv_sg8_i8_f32")
    else:
        native.check(native.lib().rwkvb_gemv_f32(y.data_ptr(), ctypes.byref(w.desc), xv.data_ptr(), _stream()),
                     "rwkvb_gemv_f32")
    torch.cuda.current_stream().synchronize() if keep else None
    return y


def lut2_tmix_gemv_batched(blobs, xs, *, out_features: int, in_features: int):
    """Four attention maps (r, k, v, o) with distinct inputs in one launch, any
    packed kind (SG8, grouped or per-tensor LUT2)."""
    if isinstance(xs, torch.Tensor):
        xs = (xs, xs, xs, xs)
    keep: list = []
    ws = [_resident(b, out_features, in_features, keep) for b in blobs[:4]]
    xv = [_vec(x, in_features) for x in xs]
    y = torch.empty((4, out_features), dtype=torch.float32, device=_dev())
    wp = (ctypes.POINTER(native.Packed) * 4)(*[ctypes.pointer(w.desc) for w in ws])
    xp = (ctypes.c_void_p * 4)(*[x.data_ptr() for x in xv])
    native.check(native.lib().rwkvb_tmix_gemv_f32(y.data_ptr(), wp, xp, 4, _stream()), "rwkvb_tmix_gemv_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return y[0], y[1], y[2], y[3]


def lut2_layer_gather(blobs, shapes) -> list[torch.Tensor]:
    """Decode several packed tensors (``lut2_layer_gather_export``,
    lut2_gather.c:135-171): one bit-exact fp32 tensor per blob."""
    return [decode_packed(b, int(s[0]), int(s[1])) for b, s in zip(blobs, shapes)]


def lut2_linear_forward(weight_blob, x: torch.Tensor, shape: tuple[int, ...]) -> torch.Tensor:
    """``x @ W.T`` for a packed ``W [out, in]`` (``lut_gemm_fused.py:1820-1851``).

    1-D ``x`` is one GEMV.  2-D ``x [batch, in]`` with an SG8 ``W`` (batch <= 64)
    runs the tcgen05 batched product (``rwkvb_gemm_sg8_f32``); other 2-D cases
    run one GEMV per row."""
    if len(shape) != 2:
        raise ValueError("lut2_linear_forward expects a 2-D weight shape")
    out_f, in_f = int(shape[0]), int(shape[1])
    if x.dim() == 1:
        return lut2_gemv(weight_blob, x, out_features=out_f, in_features=in_f)
    if x.dim() != 2 or x.shape[1] != in_f:
        raise ValueError(f"x shape {tuple(x.shape)} does not match in_features {in_f}")
    keep: list = []
    w = _resident(weight_blob, out_f, in_f, keep)
    nb = int(x.shape[0])
    if w.codec == "sg8" and 1 <= nb <= 64 and out_f % 128 == 0 and in_f % 128 == 0:
        xv = x.detach().to(device=_dev(), dtype=torch.float32).contiguous()
        y = torch.empty((nb, out_f), dtype=torch.float32, device=_dev())
        err = torch.zeros(1, dtype=torch.int32, device=_dev())
        native.check(native.lib().rwkvb_gemm_sg8_f32(y.data_ptr(), ctypes.byref(w.desc), xv.data_ptr(), nb,
                                                     err.data_ptr(), _stream()), "rwkvb_gemm_sg8_f32")
        if int(err.item()) != 0:
            native.check(native.RWKVB_ETIMEOUT, "rwkvb_gemm_sg8_f32 (device wait)")
        return y
    rows = [lut2_gemv(w, x[i], out_features=out_f, in_features=in_f) for i in range(nb)]
    if keep:
        torch.cuda.current_stream().synchronize()
    return torch.stack(rows)


def lut2_tmix_qkv_gemv_batched(blobs, xs, *, out_features: int, in_features: int):
    """Three attention projections (r, k, v) with distinct inputs in one launch."""
    if isinstance(xs, torch.Tensor):
        xs = (xs, xs, xs)
    keep: list = []
    ws = [_resident(b, out_features, in_features, keep) for b in blobs[:3]]
    xv = [_vec(x, in_features) for x in xs]
    y = torch.empty((3, out_features), dtype=torch.float32, device=_dev())
    wp = (ctypes.POINTER(native.Packed) * 3)(*[ctypes.pointer(w.desc) for w in ws])
    xp = (ctypes.c_void_p * 3)(*[x.data_ptr() for x in xv])
    if not all(_magic(b) == SG8_MAGIC for b in blobs[:3]):
        # LUT2 attention maps (grouped or per-tensor): one batched launch
        native.check(native.lib().rwkvb_tmix_gemv_f32(y.data_ptr(), wp, xp, 3, _stream()), "rwkvb_tmix_gemv_f32")
    elif activation_int8_enabled():
        native.check(native.lib().rwkvb_tmix_qkv_i8_gemv_f32(y.data_ptr(), wp, xp, _stream()),
                     "rwkvb_tmix_qkv_i8_gemv_f32")
    else:
        native.check(native.lib().rwkvb_tmix_qkv_gemv_f32(y.data_ptr(), wp, xp, _stream()),
                     "rwkvb_tmix_qkv_gemv_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return y[0], y[1], y[2]


def grouped_u8_transposed_gemv(weight_blob, x: torch.Tensor, *, out_features: int,
                               in_features: int) -> torch.Tensor:
    """``y = x @ W`` for a row-major SG8 ``W [in_features, out_features]``."""
    if _magic(weight_blob) != SG8_MAGIC:
        raise ValueError("grouped_u8_transposed_gemv requires an SG8 blob")
    keep: list = []
    w = _resident(weight_blob, in_features, out_features, keep)
    xv = _vec(x, in_features)
    y = torch.empty(out_features, dtype=torch.float32, device=_dev())
    native.check(native.lib().rwkvb_transposed_gemv_f32(y.data_ptr(), ctypes.byref(w.desc), xv.data_ptr(),
                                                        _stream()), "rwkvb_transposed_gemv_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return y


def grouped_u8_transposed_tmix_fused(blobs, xs, shapes, a0: torch.Tensor):
    """Fused TMix adapters; ``blobs`` = w1,w2,a1,a2,g1,g2[,v1,v2] (``x @ W``
    layout), ``xs`` = xw,xa,xg[,xv].  Returns ``(w, a, g[, v])``."""
    if len(blobs) not in (6, 8) or len(xs) != (4 if len(blobs) == 8 else 3):
        raise ValueError("fused TMix adapter batch has an invalid width")
    if len(shapes) != len(blobs):
        raise ValueError("fused TMix adapter shapes do not match blobs")
    if any(_magic(b) != SG8_MAGIC for b in blobs):
        raise ValueError("fused TMix adapters require grouped-U8 blobs")
    keep: list = []
    ws = [_resident(b, int(s[0]), int(s[1]), keep) for b, s in zip(blobs, shapes)]
    n_embd = int(shapes[1][1])
    xv = [_vec(x, int(shapes[2 * i][0]), f"TMix adapter input {i}") for i, x in enumerate(xs)]
    a0v = _vec(a0, n_embd, "TMix a0")
    has_v = len(blobs) == 8
    outs = [torch.empty(n_embd, dtype=torch.float32, device=_dev()) for _ in range(4 if has_v else 3)]
    descs = [w.desc for w in ws] + [ws[0].desc] * (8 - len(ws))
    wp = (ctypes.POINTER(native.Packed) * 8)(*[ctypes.pointer(d) for d in descs])
    xptrs = [x.data_ptr() for x in xv] + [xv[0].data_ptr()] * (4 - len(xv))
    xp = (ctypes.c_void_p * 4)(*xptrs)
    native.check(native.lib().rwkvb_tmix_adapters_f32(outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
                                                      outs[3].data_ptr() if has_v else None, wp, xp, a0v.data_ptr(),
                                                      int(has_v), _stream()), "rwkvb_tmix_adapters_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return tuple(outs)


def grouped_u8_cmix_gemv(key_blob, value_blob, x: torch.Tensor, *, key_out_features: int, key_in_features: int,
                         value_out_features: int, value_in_features: int) -> torch.Tensor:
    """``value @ relu(key @ x)^2`` for SG8 key/value matrices."""
    if _magic(key_blob) != SG8_MAGIC or _magic(value_blob) != SG8_MAGIC:
        raise ValueError("grouped_u8_cmix_gemv requires SG8 blobs")
    keep: list = []
    kw = _resident(key_blob, key_out_features, key_in_features, keep)
    vw = _resident(value_blob, value_out_features, value_in_features, keep)
    xv = _vec(x, key_in_features, "x")
    y = torch.empty(value_out_features, dtype=torch.float32, device=_dev())
    native.check(native.lib().rwkvb_cmix_gemv_f32(y.data_ptr(), ctypes.byref(kw.desc), ctypes.byref(vw.desc),
                                                  xv.data_ptr(), _stream()), "rwkvb_cmix_gemv_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return y


def decode_packed(weight_blob, rows: int, cols: int) -> torch.Tensor:
    """Bit-exact fp32 decode of a packed tensor in checkpoint order ``[rows, cols]``."""
    keep: list = []
    w = _resident(weight_blob, rows, cols, keep)
    out = torch.empty((rows, cols), dtype=torch.float32, device=_dev())
    native.check(native.lib().rwkvb_dequant_f32(out.data_ptr(), ctypes.byref(w.desc), _stream()),
                 "rwkvb_dequant_f32")
    if keep:
        torch.cuda.current_stream().synchronize()
    return out


def wkv7(state: torch.Tensor, r, w, k, v, kk, a, *, decay_mode: int = 0) -> torch.Tensor:
    """WKV7 update of ``state [B, H, 64, 64]`` in place; returns ``y [B, H*64]``."""
    if state.dtype != torch.float32 or not state.is_cuda or not state.is_contiguous():
        raise ValueError("state must be a contiguous fp32 CUDA tensor")
    B, H, N, _ = state.shape
    vecs = [t.reshape(B, H * N).to(device=state.device, dtype=torch.float32).contiguous() for t in (r, w, k, v, kk, a)]
    y = torch.empty((B, H * N), dtype=torch.float32, device=state.device)
    native.check(native.lib().rwkvb_wkv7_f32(state.data_ptr(), y.data_ptr(), *[t.data_ptr() for t in vecs],
                                             B, H, N, int(decay_mode), _stream()), "rwkvb_wkv7_f32")
    return y
