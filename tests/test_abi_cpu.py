"""CPU-side checks of the C ABI: the library loads without a GPU, exports every
symbol ``include/rwkv_b200.h`` declares, and its host-side validation behaves
like the reference decoders (no device work is launched here)."""

from __future__ import annotations

import ctypes
import re
import struct
from pathlib import Path

import pytest

from conftest import REPO, cases, load_golden
from rwkv_b200 import native

HEADER = REPO / "include" / "rwkv_b200.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(rwkvb_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = native.lib()
    declared = _declared_functions()
    assert "rwkvb_gemv_f32" in declared and "rwkvb_engine_create" in declared
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.rwkvb_version() == 1


def test_python_bindings_cover_the_header():
    native.lib()
    assert set(_declared_functions()) == set(native.EXPORTS)


def test_library_is_built_for_sm100a_only():
    src = (REPO / "ssd-rwkv-engine_b200" / "rwkv_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in src
    assert Path(native.native_lib_path()).is_file()


def _init(header: bytes, nbytes: int, rows: int, cols: int):
    d = native.Packed()
    st = native.lib().rwkvb_packed_init(ctypes.byref(d), header, nbytes, 0x1000, rows, cols)
    return st, d


def test_packed_init_accepts_reference_blobs():
    g = load_golden("codec_sg8.npz")
    for c in cases(g):
        blob = g[f"{c}/blob"].tobytes()
        x = g[f"{c}/input"]
        rows, cols = (x.shape if x.ndim == 2 else (1, x.size))
        st, d = _init(blob[:8], len(blob), rows, cols)
        assert st == native.RWKVB_OK, c
        assert d.kind == native.KIND_SG8 and d.group_size == int(g[f"{c}/group"])
    g = load_golden("codec_lut2.npz")
    for c in cases(g):
        blob = g[f"{c}/blob"].tobytes()
        rows, cols = g[f"{c}/input"].shape
        st, d = _init(blob[:8], len(blob), rows, cols)
        assert st == native.RWKVB_OK, c
        assert d.kind == blob[3]


def test_packed_init_rejects_malformed_blobs_like_the_reference_decoder():
    good = b"SG8\x01" + struct.pack("<I", 128)
    rows, cols = 4, 256
    n = 8 + (rows * cols // 128) * 8 + rows * cols
    assert _init(good, n, rows, cols)[0] == native.RWKVB_OK
    assert _init(good, n - 1, rows, cols)[0] == native.RWKVB_EARG           # length mismatch
    assert _init(good, n + 1, rows, cols)[0] == native.RWKVB_EARG
    assert _init(b"SG8\x02" + good[4:], n, rows, cols)[0] == native.RWKVB_EARG  # bad magic
    assert _init(b"SG8\x01" + struct.pack("<I", 0), n, rows, cols)[0] == native.RWKVB_EARG  # zero group
    assert _init(good, n, 0, cols)[0] == native.RWKVB_EARG
    # per-tensor LUT2 (TR2\x01): magic + fp32 codebook[4] + codes; its own kind id
    tensor = b"TR2\x01" + struct.pack("<f", 0.0)  # codebook[0] = 0.0 is not a zero group size
    need = 20 + (rows * cols + 3) // 4
    st, d = _init(tensor, need, rows, cols)
    assert st == native.RWKVB_OK and d.kind == native.KIND_LUT2_TENSOR and d.group_size == rows * cols
    assert _init(tensor, need - 1, rows, cols)[0] == native.RWKVB_EARG
    assert _init(b"TR2\x02" + good[4:], need, rows, cols)[0] == native.RWKVB_EARG  # FLUTE rows: not a device kind
    short = 8 + (rows * cols // 64) * 8 + rows * cols // 4 - 1
    assert _init(b"TR2\x04" + struct.pack("<I", 64), short, rows, cols)[0] == native.RWKVB_EARG


def test_status_strings():
    lib = native.lib()
    for st in range(6):
        assert lib.rwkvb_status_string(st)
    err = native.RwkvbError(native.RWKVB_EARG, "x")
    assert "invalid argument" in str(err)


def test_null_arguments_rejected_without_a_device():
    lib = native.lib()
    assert lib.rwkvb_gemv_f32(None, None, None, None) == native.RWKVB_EARG
    assert lib.rwkvb_dequant_f32(None, None, None) == native.RWKVB_EARG
    assert lib.rwkvb_engine_create(None, 0, None) == native.RWKVB_EARG
    assert lib.rwkvb_engine_destroy(None) == native.RWKVB_EARG
    assert lib.rwkvb_wkv7_f32(None, None, None, None, None, None, None, None, 1, 1, 64, 0, None) == native.RWKVB_EARG
