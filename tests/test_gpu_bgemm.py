"""GPU parity of the batched SG8 product on the tcgen05 tensor cores
(``rwkvb_gemm_sg8_f32`` through ``lut2_linear_forward``).

The reference's batched branch decodes W and calls ``torch.nn.functional.linear``
(``rwkv_ssd/runtime/lut_gemm_fused.py:1820-1851``); here the bar is a float64
product of the bit-exact decoded weights, rtol/atol 2e-5 (the same bar as the
GEMV family), plus run-to-run determinism.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle import codec as oc  # noqa: E402
from rwkv_b200 import lut_gemm_fused as lg  # noqa: E402
from rwkv_b200 import native  # noqa: E402
from rwkv_b200 import synth  # noqa: E402

TOL = dict(rtol=2e-5, atol=2e-5)


def _case(rows: int, cols: int, group: int, batch: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn((rows, cols), generator=gen) * 0.02
    x = torch.randn((batch, cols), generator=gen)
    blob = synth.encode_sg8(w.cuda(), group).cpu().numpy().tobytes()
    dec = torch.from_numpy(oc.decode_sg8(blob, rows * cols).reshape(rows, cols)).cuda().double()
    exact = (x.cuda().double() @ dec.T).cpu().numpy()
    return blob, x, exact


@pytest.mark.parametrize("rows,cols,group,batch", [
    (128, 128, 128, 1),
    (256, 512, 128, 8),
    (384, 256, 64, 5),
    (2560, 2560, 128, 64),
    (10240, 2560, 128, 64),
    (2560, 10240, 128, 64),
    (2560, 2560, 128, 33),
])
def test_gemm_sg8_matches_float64(rows, cols, group, batch):
    blob, x, exact = _case(rows, cols, group, batch, rows * 7 + cols + batch)
    y = lg.lut2_linear_forward(blob, x, (rows, cols))
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), exact, **TOL)


def test_gemm_sg8_head_shape_and_determinism():
    rows, cols, batch = 65536, 2560, 64
    blob, x, exact = _case(rows, cols, 128, batch, 11)
    y1 = lg.lut2_linear_forward(blob, x, (rows, cols))
    y2 = lg.lut2_linear_forward(blob, x, (rows, cols))
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    np.testing.assert_allclose(y1.cpu().numpy(), exact, **TOL)
    # greedy ids of every session equal those of the exact product
    assert np.array_equal(y1.argmax(dim=1).cpu().numpy(), exact.argmax(axis=1))


def test_gemm_sg8_batch1_agrees_with_gemv():
    blob, x, _ = _case(2560, 2560, 128, 1, 3)
    y = lg.lut2_linear_forward(blob, x, (2560, 2560))
    g = lg.lut2_gemv(blob, x[0], out_features=2560, in_features=2560)
    np.testing.assert_allclose(y[0].cpu().numpy(), g.cpu().numpy(), **TOL)


def test_gemm_sg8_rejects_unsupported_shapes():
    blob, x, _ = _case(200, 256, 128, 2, 5)  # rows not a multiple of 128: per-row GEMV path
    y = lg.lut2_linear_forward(blob, x, (200, 256))
    assert y.shape == (2, 200)
    from rwkv_b200.residency import WeightArena

    arena = WeightArena([("w", blob, (200, 256), "sg8")], torch.device("cuda", 0))
    out = torch.empty((2, 200), device="cuda")
    st = native.lib().rwkvb_gemm_sg8_f32(out.data_ptr(), native.ctypes.byref(arena["w"].desc),
                                         x.cuda().data_ptr(), 2, None, None)
    assert st == native.RWKVB_EUNSUPPORTED
    st = native.lib().rwkvb_gemm_sg8_f32(out.data_ptr(), native.ctypes.byref(arena["w"].desc),
                                         x.cuda().data_ptr(), 65, None, None)
    assert st == native.RWKVB_EARG
