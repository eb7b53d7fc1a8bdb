"""Oracle restatement of the pack codecs on the decode hot path (NumPy, CPU).

Test infrastructure: see ``oracle/__init__.py``.  Every function names the
reference source it restates.  Arithmetic is kept in the same dtype and the
same operation order as the reference so that encoded bytes and decoded
values are bit-identical (checked against ``tests/golden`` vectors produced
by the reference itself).

Wire formats
------------
``SG8\\x01`` grouped affine UINT8 (reference ``pack_codec.py:13-68``)::

    b"SG8\\x01" | u32 group_size | f32[groups][2] (min, max) | u8[numel]

Groups run over the row-major flattened tensor; the final group may be
partial.  Dequant: ``delta = (max - min) * f32(1/255)``; ``w = q * delta + min``
(two roundings, no fused multiply-add; ``pack_codec.py:174-182``).

Grouped LUT2 (reference ``trinity_codec.py:52-58``, ``:446-623``)::

    b"TR2" + kind | u32 group_size | records[groups] | 2-bit codes (LSB first)

``kind`` 3: 16-byte records of four fp32 centroids; 4 / 6: 8-byte records
of four fp16 centroids; 5 / 7: 16-byte records ``f16[4] centroids, u8[2]
residual positions, f16[2] residual deltas, u8[2] reserved``.  Kinds 6 and 7
store the tensor transposed (input-major logical order).
"""

from __future__ import annotations

import struct

import numpy as np

SG8_MAGIC = b"SG8\x01"
LUT2_GROUPED = b"TR2\x03"
LUT2_GROUPED_FP16 = b"TR2\x04"
LUT2_GROUPED_RESIDUAL = b"TR2\x05"
LUT2_INPUT_FP16 = b"TR2\x06"
LUT2_INPUT_RESIDUAL = b"TR2\x07"
LUT2_GROUPED_KINDS = (
    LUT2_GROUPED,
    LUT2_GROUPED_FP16,
    LUT2_GROUPED_RESIDUAL,
    LUT2_INPUT_FP16,
    LUT2_INPUT_RESIDUAL,
)

_INV255 = np.float32(1.0 / 255.0)


# --------------------------------------------------------------------------
# SG8 grouped affine UINT8
# --------------------------------------------------------------------------
def encode_sg8(values: np.ndarray, group_size: int = 128) -> bytes:
    """Restates ``encode_scale_u8_grouped`` (``pack_codec.py:33-68``)."""
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    flat = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    groups = (flat.size + group_size - 1) // group_size
    mins = np.empty(groups, dtype=np.float32)
    maxs = np.empty(groups, dtype=np.float32)
    quant = np.empty(flat.size, dtype=np.uint8)
    batch = max(1, 1_000_000 // group_size)
    for first in range(0, groups, batch):
        count = min(batch, groups - first)
        start = first * group_size
        avail = min(count * group_size, flat.size - start)
        chunk = np.empty((count, group_size), dtype=np.float32)
        chunk.reshape(-1)[:avail] = flat[start : start + avail]
        if avail < count * group_size:
            # The partial final group is padded with its last value.
            chunk.reshape(-1)[avail:] = chunk.reshape(-1)[avail - 1]
        lo = chunk.min(axis=1)
        hi = chunk.max(axis=1)
        hi = np.where(hi - lo < 1e-12, lo + 1.0, hi).astype(np.float32)
        mins[first : first + count] = lo
        maxs[first : first + count] = hi
        q = np.rint((chunk - lo[:, None]) / (hi - lo)[:, None] * 255.0)
        q = q.clip(0, 255).astype(np.uint8)
        quant[start : start + avail] = q.reshape(-1)[:avail]
    scales = np.stack((mins, maxs), axis=1)
    return SG8_MAGIC + struct.pack("<I", group_size) + scales.tobytes() + quant.tobytes()


def sg8_parse(blob: bytes | memoryview, numel: int) -> tuple[int, np.ndarray, np.ndarray]:
    """Split an SG8 blob into (group_size, scales[groups, 2], quant[numel]).

    Validation follows ``decode_scale_u8_grouped_to_tensor``
    (``pack_codec.py:126-137``): wrong magic, zero group size or a length that
    is not exactly ``8 + groups*8 + numel`` raise ``ValueError``.
    """
    if len(blob) < 8 or bytes(blob[:4]) != SG8_MAGIC:
        raise ValueError("bad scale_u8_grouped blob")
    (g,) = struct.unpack("<I", bytes(blob[4:8]))
    if g <= 0:
        raise ValueError("invalid scale_u8_grouped size")
    groups = (numel + g - 1) // g
    end = 8 + groups * 8
    if len(blob) != end + numel:
        raise ValueError("scale_u8_grouped length mismatch")
    scales = np.frombuffer(blob, dtype=np.float32, offset=8, count=groups * 2).reshape(groups, 2)
    quant = np.frombuffer(blob, dtype=np.uint8, offset=end, count=numel)
    return g, scales, quant


def decode_sg8(blob: bytes | memoryview, numel: int) -> np.ndarray:
    """Restates ``_decode_grouped_u8_values`` (``pack_codec.py:147-183``).

    ``delta = (max - min) * f32(1/255)`` then ``q * delta + min`` in fp32 with
    two separate roundings.
    """
    g, scales, quant = sg8_parse(blob, numel)
    out = np.empty(numel, dtype=np.float32)
    if numel == 0:
        return out
    full, rem = divmod(numel, g)
    if full:
        q = quant[: full * g].astype(np.float32).reshape(full, g)
        o = out[: full * g].reshape(full, g)
        delta = (scales[:full, 1] - scales[:full, 0]) * _INV255
        np.multiply(q, delta[:, None], out=o)
        np.add(o, scales[:full, 0, None], out=o)
    if rem:
        mn = scales[full, 0]
        delta = (scales[full, 1] - mn) * _INV255
        out[full * g :] = mn + quant[full * g :].astype(np.float32) * delta
    return out


# --------------------------------------------------------------------------
# Grouped LUT2
# --------------------------------------------------------------------------
def pack_2bit(indices: np.ndarray) -> bytes:
    """Restates ``_pack_2bit`` (``trinity_codec.py:239-251``): 4 codes/byte, LSB first."""
    idx = indices.astype(np.uint8).ravel()
    pad = (4 - idx.size % 4) % 4
    if pad:
        idx = np.append(idx, np.zeros(pad, dtype=np.uint8))
    out = (idx[0::4] & 3) | ((idx[1::4] & 3) << 2) | ((idx[2::4] & 3) << 4) | ((idx[3::4] & 3) << 6)
    return out.astype(np.uint8).tobytes()


def unpack_2bit(data: bytes | memoryview, numel: int) -> np.ndarray:
    """Restates ``_unpack_2bit`` (``trinity_codec.py:276-303``)."""
    packed = np.frombuffer(data, dtype=np.uint8)
    need = (numel + 3) // 4
    if packed.size < need:
        raise ValueError("trinity_lut2 indices short")
    packed = packed[:need]
    shifts = np.array([0, 2, 4, 6], dtype=np.uint8)
    codes = (packed[:, None] >> shifts[None, :]) & 3
    return codes.reshape(-1)[:numel].astype(np.uint8)


def kmeans_codebooks(values: np.ndarray, group_size: int, iters: int = 12) -> np.ndarray:
    """Restates ``codebooks_groupwise_kmeans`` (``trinity_codebook.py:139-195``).

    Quantile-initialised batched 1-D Lloyd iterations, four centroids per
    contiguous group, sorted ascending.
    """
    k = 4
    vals = np.asarray(values, dtype=np.float32).reshape(-1)
    groups = (vals.size + group_size - 1) // group_size
    out = np.empty((groups, k), dtype=np.float32)
    quantiles = np.linspace(0.0, 1.0, k + 2, dtype=np.float64)[1:-1]
    batch = max(1, min(4096, 2_000_000 // group_size))
    for first in range(0, groups, batch):
        count = min(batch, groups - first)
        start = first * group_size
        avail = min(count * group_size, vals.size - start)
        chunk = np.empty((count, group_size), dtype=np.float32)
        src = vals[start : start + avail]
        chunk.reshape(-1)[:avail] = src
        valid = np.arange(count * group_size).reshape(count, group_size) < avail
        if avail < count * group_size:
            chunk.reshape(-1)[avail:] = src[-1] if avail else 0.0
        centers = np.quantile(chunk, quantiles, axis=1).T.astype(np.float32)
        for _ in range(max(1, int(iters))):
            labels = np.abs(chunk[:, :, None] - centers[:, None, :]).argmin(axis=2)
            updated = centers.copy()
            for j in range(k):
                sel = (labels == j) & valid
                cnt = sel.sum(axis=1)
                sums = np.where(sel, chunk, 0.0).sum(axis=1, dtype=np.float64)
                present = cnt > 0
                updated[present, j] = (sums[present] / cnt[present]).astype(np.float32)
            updated.sort(axis=1)
            if np.max(np.abs(updated - centers)) < 1e-7:
                centers = updated
                break
            centers = updated
        out[first : first + count] = centers
    return out


def lut2_assign(values: np.ndarray, codebooks: np.ndarray, group_size: int) -> np.ndarray:
    """Restates ``_indices_groupwise`` (``trinity_codec.py:98-115``): nearest centroid, first on ties."""
    flat = np.asarray(values, dtype=np.float32).reshape(-1)
    out = np.empty(flat.size, dtype=np.uint8)
    groups = codebooks.shape[0]
    batch = max(1, 1_000_000 // group_size)
    for first in range(0, groups, batch):
        count = min(batch, groups - first)
        start = first * group_size
        avail = min(count * group_size, flat.size - start)
        v = flat[start : start + avail]
        gid = np.arange(avail, dtype=np.intp) // group_size
        local = codebooks[first : first + count]
        out[start : start + avail] = np.abs(v[:, None] - local[gid]).argmin(axis=1).astype(np.uint8)
    return out


def encode_lut2_grouped(
    tensor: np.ndarray, group_size: int = 64, *, kind: bytes = LUT2_GROUPED_FP16
) -> bytes:
    """Restates ``encode_trinity_lut2`` for the k-means grouped kinds.

    ``kind`` ``TR2\\x04`` (``groupwise_kmeans_fp16``), ``TR2\\x06``
    (``groupwise_input_fp16``: the 2-D tensor is transposed first),
    ``TR2\\x03`` (``groupwise_kmeans``, fp32 records) and the residual kinds
    ``TR2\\x05`` / ``TR2\\x07`` (``groupwise_kmeans_residual`` /
    ``groupwise_input_residual``: 16-byte records of the fp16 codebook, the
    two in-group positions of largest |residual| and their fp16 residuals,
    ``_residual_metadata``, ``trinity_codec.py:162-217``); see
    ``trinity_codec.py:494-623``.
    """
    t = np.asarray(tensor, dtype=np.float32)
    if kind in (LUT2_INPUT_FP16, LUT2_INPUT_RESIDUAL) and t.ndim == 2:
        flat = np.ascontiguousarray(t.T).reshape(-1)
    elif kind in LUT2_GROUPED_KINDS:
        flat = t.reshape(-1)
    else:
        raise ValueError(f"not a grouped LUT2 kind: {kind!r}")
    cb = kmeans_codebooks(flat, group_size)
    if kind != LUT2_GROUPED:
        cb = cb.astype(np.float16).astype(np.float32)
    idx = lut2_assign(flat, cb, group_size)
    head = kind + struct.pack("<I", group_size)
    if kind == LUT2_GROUPED:
        return head + cb.astype(np.float32).tobytes() + pack_2bit(idx)
    if kind in (LUT2_GROUPED_RESIDUAL, LUT2_INPUT_RESIDUAL):
        return head + _residual_records(flat, cb.astype(np.float16), idx, group_size) + pack_2bit(idx)
    return head + cb.astype(np.float16).tobytes() + pack_2bit(idx)


def _residual_records(flat: np.ndarray, cb16: np.ndarray, idx: np.ndarray, g: int) -> bytes:
    """16-byte residual records: fp16 codebook[4], u8 positions[2] of the two
    largest |value - codebook value| in the group, their fp16 residuals, two
    reserved bytes."""
    groups = cb16.shape[0]
    rec = np.zeros(groups, dtype=np.dtype([("cb", "<f2", (4,)), ("pos", "u1", (2,)), ("dlt", "<f2", (2,)),
                                           ("pad", "u1", (2,))]))
    rec["cb"] = cb16
    padded = np.zeros(groups * g, dtype=np.float32)
    gid = np.arange(flat.size) // g
    padded[:flat.size] = flat - cb16.astype(np.float32)[gid, idx]
    res = padded.reshape(groups, g)
    pos = np.argpartition(np.abs(res), -2, axis=1)[:, -2:] if g > 1 else np.zeros((groups, 2), np.intp)
    rec["pos"] = pos.astype(np.uint8)
    rec["dlt"] = np.take_along_axis(res, pos, axis=1).astype(np.float16)
    return rec.tobytes()


def encode_lut2_tensor(tensor: np.ndarray, iters: int = 12) -> bytes:
    """A per-tensor LUT2 blob (``TR2\\x01``): one fp32 codebook of four k-means
    centroids for the whole tensor and its flattened 2-bit codes
    (``trinity_codec.py:612-625``)."""
    flat = np.asarray(tensor, dtype=np.float32).reshape(-1)
    cb = kmeans_codebooks(flat, flat.size, iters)
    idx = lut2_assign(flat, cb, flat.size)
    return b"TR2\x01" + cb.reshape(-1).astype(np.float32).tobytes() + pack_2bit(idx)


def lut2_record_bytes(kind: bytes) -> int:
    """Record size per group (``trinity_codec.py:779-784``)."""
    if kind in (LUT2_GROUPED_RESIDUAL, LUT2_INPUT_RESIDUAL):
        return 16
    if kind in (LUT2_GROUPED_FP16, LUT2_INPUT_FP16):
        return 8
    if kind == LUT2_GROUPED:
        return 16
    raise ValueError(f"not a grouped LUT2 kind: {kind!r}")


def decode_lut2_grouped(blob: bytes | memoryview, shape: tuple[int, ...]) -> np.ndarray:
    """Restates ``decode_trinity_lut2_to_tensor`` for grouped kinds
    (``trinity_codec.py:769-885``) and ``_decode_grouped_lut2_cpu``
    (``:381-438``).  Returns fp32 values in the logical ``shape``.
    """
    numel = int(np.prod(shape)) if len(shape) else 1
    if len(blob) < 8:
        raise ValueError("grouped trinity_lut2 blob too short")
    kind = bytes(blob[:4])
    if kind not in LUT2_GROUPED_KINDS:
        raise ValueError("not a grouped LUT2 blob")
    (g,) = struct.unpack("<I", bytes(blob[4:8]))
    if g <= 0:
        raise ValueError("invalid grouped trinity_lut2 group size")
    groups = (numel + g - 1) // g
    rec = lut2_record_bytes(kind)
    cb_end = 8 + groups * rec
    if len(blob) < cb_end + (numel + 3) // 4:
        raise ValueError("grouped trinity_lut2 payload short")
    buf = bytes(blob)
    if kind == LUT2_GROUPED:
        cb = np.frombuffer(buf, dtype=np.float32, offset=8, count=groups * 4).reshape(groups, 4)
    else:
        cb = np.ndarray((groups, 4), dtype=np.float16, buffer=buf, offset=8,
                        strides=(rec, 2)).astype(np.float32)
    idx = unpack_2bit(memoryview(buf)[cb_end:], numel)
    flat = np.empty(numel, dtype=np.float32)
    gid = np.arange(numel, dtype=np.intp) // g
    flat[:] = cb[gid, idx]
    if kind in (LUT2_GROUPED_RESIDUAL, LUT2_INPUT_RESIDUAL):
        pos = np.ndarray((groups, 2), dtype=np.uint8, buffer=buf, offset=16, strides=(rec, 1))
        dlt = np.ndarray((groups, 2), dtype=np.float16, buffer=buf, offset=18,
                         strides=(rec, 2)).astype(np.float32)
        absolute = np.arange(groups, dtype=np.intp)[:, None] * g + pos.astype(np.intp)
        ok = absolute < numel
        flat[absolute[ok]] += dlt[ok]
    if kind in (LUT2_INPUT_FP16, LUT2_INPUT_RESIDUAL) and len(shape) == 2:
        return np.ascontiguousarray(flat.reshape(shape[1], shape[0]).T)
    return flat.reshape(shape)


def decode_lut2_tensor(blob: bytes | memoryview, numel: int) -> np.ndarray:
    """Restates the per-tensor LUT2 (``TR2\\x01``) decode: ``lut2_gather_packed``
    (``lut2_gather.c:81-105``) over the flattened codes after the fp32
    codebook (``trinity_codec.py:306-323``)."""
    buf = bytes(blob)
    if buf[:4] != b"TR2\x01" or len(buf) < 20 + (numel + 3) // 4:
        raise ValueError("not a per-tensor LUT2 blob")
    cb = np.frombuffer(buf, dtype=np.float32, offset=4, count=4)
    return cb[unpack_2bit(memoryview(buf)[20:], numel)].astype(np.float32)
