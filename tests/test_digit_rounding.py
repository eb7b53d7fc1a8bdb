"""The digit kernels round with the 1.5 * 2^23 shift instead of ``rintf`` and a
float->int conversion (``csrc/imma.cuh`` ``emit_digits``, ``csrc/bgemm.cuh``
``bg_emit_group``).  This checks the identity they rely on, in fp32 with
round-to-nearest-even: for |y| <= 127, ``(y + 1.5*2^23) - 1.5*2^23 == rint(y)``
and the low byte of the sum's bit pattern is rint(y) as a two's-complement byte,
ties included."""

import numpy as np

SHIFT = np.float32(12582912.0)


def test_shift_rounding_equals_rint_with_ties():
    rng = np.random.default_rng(0)
    y = np.concatenate([
        rng.uniform(-127.0, 127.0, 200000).astype(np.float32),
        (np.arange(-127, 127, dtype=np.float32) + np.float32(0.5)),  # exact ties
        np.array([-127.0, 127.0, 0.0, -0.0, 0.49999997, -0.49999997, 126.5, -126.5], dtype=np.float32),
    ])
    s = (y + SHIFT).astype(np.float32)
    x = (s - SHIFT).astype(np.float32)
    assert np.array_equal(x, np.rint(y).astype(np.float32))
    low = (s.view(np.uint32) & 0xFF).astype(np.uint8)
    assert np.array_equal(low, np.rint(y).astype(np.int32).astype(np.int8).view(np.uint8))
    # the batched digits are stored offset by 127
    off = ((s.view(np.uint32) + 127) & 0xFF).astype(np.int32)
    assert np.array_equal(off, np.rint(y).astype(np.int32) + 127)
