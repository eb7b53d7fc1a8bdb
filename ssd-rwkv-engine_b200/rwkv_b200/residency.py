"""HBM residency for packed weights.

The reference streams packed layers from SSD through pinned staging buffers
(``rwkv_ssd/runtime/staging.py:40-129``) and keeps the raw blob views in its
provider (``weight_provider.py:780-907``).  Here every blob of a pack is
copied once, unchanged, into one device arena:

* blobs are placed so that their code payload starts on a 16-byte boundary
  (the vectorised GEMV paths read it with 16-byte loads) and their header on
  an 8-byte boundary;
* host blobs go through a reusable pinned staging buffer and are copied with
  ``cudaMemcpyAsync`` on a side stream, so upload overlaps encoding/IO;
* fp32 skeleton vectors live in a second arena; packed 1-D/2-D skeleton
  tensors that the reference provider decodes densely (``r_k``) are decoded on
  the device with the bit-exact dequant kernel.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass

import numpy as np
import torch

from . import native

_ALIGN = 256


def _blob_header(payload) -> bytes:
    if isinstance(payload, torch.Tensor):
        return payload[:8].cpu().numpy().tobytes()
    return bytes(payload[:8])


def _blob_len(payload) -> int:
    return int(payload.numel()) if isinstance(payload, torch.Tensor) else len(payload)


def _meta_bytes(header: bytes, rows: int, cols: int) -> int:
    """Header + per-group records: the offset of the code payload in the blob."""
    (g,) = struct.unpack("<I", header[4:8])
    if g == 0:
        raise ValueError("packed blob with zero group size")
    groups = (rows * cols + g - 1) // g
    if header[:4] == b"SG8\x01":
        return 8 + groups * 8
    if header[:3] == b"TR2" and header[3] in (3, 4, 5, 6, 7):
        return 8 + groups * (8 if header[3] in (4, 6) else 16)
    raise ValueError(f"unsupported packed blob magic {header[:4]!r}")


@dataclass
class DevicePacked:
    """One packed matrix resident in HBM."""

    name: str
    desc: native.Packed
    shape: tuple[int, int]
    codec: str

    @property
    def ptr(self) -> int:
        return int(self.desc.data)


class WeightArena:
    """Device-resident copy of a set of packed blobs (one allocation)."""

    def __init__(self, items: list[tuple[str, object, tuple[int, int], str]], device: torch.device,
                 stream: torch.cuda.Stream | None = None):
        lib = native.lib()
        self.device = device
        offs: list[int] = []
        heads: list[bytes] = []
        cur = 0
        for _name, payload, shape, _codec in items:
            head = _blob_header(payload)
            meta = _meta_bytes(head, shape[0], shape[1])
            cur = (cur + _ALIGN - 1) // _ALIGN * _ALIGN
            # payload (blob + meta) 16-byte aligned; blob start stays 8-byte aligned
            cur += (16 - meta % 16) % 16
            offs.append(cur)
            heads.append(head)
            cur += _blob_len(payload)
        self.nbytes = cur
        self.buf = torch.empty(max(cur, 16), dtype=torch.uint8, device=device)
        base = self.buf.data_ptr()
        self.items: dict[str, DevicePacked] = {}
        stream = stream or torch.cuda.Stream(device=device)
        staging = None
        with torch.cuda.stream(stream):
            for (name, payload, shape, codec), off, head in zip(items, offs, heads):
                n = _blob_len(payload)
                dst = self.buf[off:off + n]
                if isinstance(payload, torch.Tensor) and payload.is_cuda:
                    dst.copy_(payload, non_blocking=True)
                else:
                    host = torch.frombuffer(bytearray(payload) if isinstance(payload, bytes) else payload,
                                            dtype=torch.uint8) if not isinstance(payload, torch.Tensor) else payload
                    if staging is None or staging.numel() < n:
                        stream.synchronize()
                        staging = torch.empty(max(n, 1 << 24), dtype=torch.uint8, pin_memory=True)
                    else:
                        stream.synchronize()
                    staging[:n].copy_(host)
                    dst.copy_(staging[:n], non_blocking=True)
                d = native.Packed()
                native.check(lib.rwkvb_packed_init(ctypes.byref(d), head, n, base + off, shape[0], shape[1]),
                             f"rwkvb_packed_init({name})")
                self.items[name] = DevicePacked(name, d, shape, codec)
        stream.synchronize()

    def __getitem__(self, name: str) -> DevicePacked:
        return self.items[name]

    def __contains__(self, name: str) -> bool:
        return name in self.items


class VectorArena:
    """fp32 skeleton vectors on the device, 16-byte aligned each."""

    def __init__(self, vecs: dict[str, np.ndarray | torch.Tensor], device: torch.device):
        sizes = {k: int(np.prod(v.shape)) if not isinstance(v, torch.Tensor) else int(v.numel())
                 for k, v in vecs.items()}
        offs, cur = {}, 0
        for k, n in sizes.items():
            offs[k] = cur
            cur += (n + 3) // 4 * 4
        self.buf = torch.zeros(max(cur, 4), dtype=torch.float32, device=device)
        self.offs = offs
        self.sizes = sizes
        self.extra: dict[str, torch.Tensor] = {}
        for k, v in vecs.items():
            t = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
            self.buf[offs[k]:offs[k] + sizes[k]].copy_(t.reshape(-1).to(torch.float32))

    def add_decoded(self, name: str, packed: DevicePacked) -> None:
        """Add the bit-exact device decode of a packed tensor (e.g. ``r_k``)."""
        n = packed.shape[0] * packed.shape[1]
        out = torch.empty(n, dtype=torch.float32, device=self.buf.device)
        st = torch.cuda.current_stream(self.buf.device)
        native.check(native.lib().rwkvb_dequant_f32(out.data_ptr(), ctypes.byref(packed.desc), st.cuda_stream),
                     f"rwkvb_dequant_f32({name})")
        self.extra[name] = out

    def ptr(self, name: str) -> int:
        if name in self.extra:
            return self.extra[name].data_ptr()
        return self.buf.data_ptr() + 4 * self.offs[name]

    def view(self, name: str) -> torch.Tensor:
        if name in self.extra:
            return self.extra[name]
        return self.buf[self.offs[name]:self.offs[name] + self.sizes[name]]
