"""rwkvb_cmix_gemv_f32_noalloc: the channel mix with its intermediate in a fixed
static device buffer instead of a per-call allocation.

Collected last on purpose (file name): it must give the same answers whether
it runs alone or after every other test has used the device.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from rwkv_b200 import native


def _sg8(rows: int, cols: int, seed: int) -> bytes:
    from oracle import codec as oc

    g = np.random.default_rng(seed)
    w = (g.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    return oc.encode_sg8(w, 128)


def _fake(rows: int, cols: int) -> native.Packed:
    # a descriptor that is never dereferenced: the call must reject it on the host
    return native.Packed(data=0x1000, bytes=8 + ((rows * cols + 127) // 128) * 8 + rows * cols, kind=1,
                         group_size=128, rows=rows, cols=cols)


def test_noalloc_rejects_oversize_before_touching_the_device():
    lib = native.lib()
    f = native.CMIX_NOALLOC_MAX_FFN + 128
    key, value = _fake(f, 256), _fake(256, f)
    st = lib.rwkvb_cmix_gemv_f32_noalloc(0x2000, ctypes.byref(key), ctypes.byref(value), 0x3000, None)
    assert st == native.RWKVB_ESCRATCH
    assert b"scratch" in lib.rwkvb_status_string(st)
    # a mismatched inner width is still an argument error
    st = lib.rwkvb_cmix_gemv_f32_noalloc(0x2000, ctypes.byref(_fake(512, 256)), ctypes.byref(_fake(256, 384)),
                                         0x3000, None)
    assert st == native.RWKVB_EARG


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("C,F", [(256, 1024), (2560, 10240)])
def test_noalloc_matches_allocating_entry_point_twice_in_a_row(C, F):
    from rwkv_b200 import lut_gemm_fused as lg

    lib = native.lib()
    keep: list = []
    kw = lg._resident(_sg8(F, C, 11), F, C, keep)
    vw = lg._resident(_sg8(C, F, 12), C, F, keep)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cpu").manual_seed(5)
    for call in range(2):
        x = torch.randn(C, generator=g).cuda()
        y_ref = torch.full((C,), float("nan"), device="cuda")
        y = torch.full((C,), float("nan"), device="cuda")
        native.check(lib.rwkvb_cmix_gemv_f32(y_ref.data_ptr(), ctypes.byref(kw.desc), ctypes.byref(vw.desc),
                                             x.data_ptr(), stream), "rwkvb_cmix_gemv_f32")
        native.check(lib.rwkvb_cmix_gemv_f32_noalloc(y.data_ptr(), ctypes.byref(kw.desc), ctypes.byref(vw.desc),
                                                     x.data_ptr(), stream), "rwkvb_cmix_gemv_f32_noalloc")
        torch.cuda.synchronize()
        # same kernels, same launch shapes: identical bits
        assert torch.equal(y, y_ref), f"call {call}: max diff {(y - y_ref).abs().max().item()}"
        assert torch.isfinite(y).all()
