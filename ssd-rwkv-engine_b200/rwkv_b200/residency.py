"""HBM residency for packed weights.

The reference streams packed layers from SSD through pinned staging buffers
(``rwkv_ssd/runtime/staging.py:40-129``) and keeps the raw blob views in its
provider (``weight_provider.py:780-907``).  Here the blobs of a pack are
copied, unchanged, into HBM:

* blobs are placed so that their code payload starts on a 16-byte boundary
  (the vectorised GEMV paths read it with 16-byte loads) and their header on
  an 8-byte boundary;
* host blobs go through a reusable pinned staging buffer and are copied with
  ``cudaMemcpyAsync`` on a side stream, so upload overlaps encoding/IO;
* fp32 skeleton vectors live in a second arena; packed 1-D/2-D skeleton
  tensors that the reference provider decodes densely (``r_k``) are decoded on
  the device with the bit-exact dequant kernel;
* under an HBM budget smaller than the model (``LayerStaging``), the layers
  that do not fit stay in pinned host memory, one contiguous image per layer,
  and are staged into a ring of device slots on every token step.
"""

from __future__ import annotations

import ctypes
import re
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
    if header[:4] == b"TR2\x01":  # per-tensor LUT2: magic + fp32 codebook[4]
        return 20
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


def _place(items) -> tuple[list[int], list[bytes], int]:
    """Offsets of blobs packed back to back: each at a 256-byte boundary plus
    the padding that puts its code payload on a 16-byte boundary."""
    offs: list[int] = []
    heads: list[bytes] = []
    cur = 0
    for _name, payload, shape, _codec in items:
        head = _blob_header(payload)
        meta = _meta_bytes(head, shape[0], shape[1])
        cur = (cur + _ALIGN - 1) // _ALIGN * _ALIGN
        # payload (blob + meta) 16-byte aligned; blob start stays 8-byte aligned
        # (4-byte for the 20-byte header of a per-tensor LUT2 blob)
        cur += (16 - meta % 16) % 16
        offs.append(cur)
        heads.append(head)
        cur += _blob_len(payload)
    return offs, heads, cur


def _host_u8(payload) -> torch.Tensor:
    if isinstance(payload, torch.Tensor):
        return payload.reshape(-1).cpu()
    return torch.frombuffer(bytearray(payload) if isinstance(payload, bytes) else payload, dtype=torch.uint8)


class WeightArena:
    """Device-resident copy of a set of packed blobs (one allocation)."""

    def __init__(self, items: list[tuple[str, object, tuple[int, int], str]], device: torch.device,
                 stream: torch.cuda.Stream | None = None):
        lib = native.lib()
        self.device = device
        offs, heads, cur = _place(items)
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


_LAYER_RE = re.compile(r"^blocks\.(\d+)\.")


def layer_of(name: str) -> int:
    """Layer index of a per-layer tensor name, -1 for global tensors."""
    m = _LAYER_RE.match(name)
    return int(m.group(1)) if m else -1


def hot_layer_order(n_layer: int) -> list[int]:
    """Layers in the order they are kept resident under a budget: outermost
    first (0, L-1, 1, L-2, ...), as the reference's partial mode keeps the
    first and last layers resident (``residency.py:98-118``)."""
    out, lo, hi = [], 0, n_layer - 1
    while lo <= hi:
        out.append(lo)
        if hi != lo:
            out.append(hi)
        lo, hi = lo + 1, hi - 1
    return out


class LayerStaging:
    """The streamed tier of a model under an HBM budget.

    Streamed layers (``streamed``, in step order) keep their packed blobs in
    pinned host memory, one image per layer (the blobs at the offsets of the
    layer's slot layout), and ``n_slots`` device slots of ``layer_bytes`` each
    receive them on every token step (``rwkvb_engine_create_staged``).
    ``descs[name]`` are the streamed matrices' descriptors, pointing into
    their layer's slot.  ``desc`` is the ``rwkvb_stage_desc``."""

    def __init__(self, layers: dict[int, list[tuple[str, object, tuple[int, int], str]]], streamed: list[int],
                 n_layer: int, n_slots: int, device: torch.device):
        lib = native.lib()
        self.streamed = list(streamed)
        self.n_slots = max(1, min(int(n_slots), len(self.streamed)))
        plans = {li: _place(layers[li]) for li in self.streamed}
        self.layer_bytes = max((p[2] for p in plans.values()), default=16)
        self.layer_bytes = (self.layer_bytes + _ALIGN - 1) // _ALIGN * _ALIGN
        self.slots = torch.empty(self.n_slots * self.layer_bytes, dtype=torch.uint8, device=device)
        self.host: dict[int, torch.Tensor] = {}
        self.descs: dict[str, DevicePacked] = {}
        slot_of = [-1] * n_layer
        for j, li in enumerate(self.streamed):
            slot = j % self.n_slots
            slot_of[li] = slot
            offs, heads, _ = plans[li]
            img = torch.zeros(self.layer_bytes, dtype=torch.uint8, pin_memory=True)
            dev_base = self.slots.data_ptr() + slot * self.layer_bytes
            for (name, payload, shape, codec), off, head in zip(layers[li], offs, heads):
                n = _blob_len(payload)
                img[off:off + n].copy_(_host_u8(payload))
                d = native.Packed()
                native.check(lib.rwkvb_packed_init(ctypes.byref(d), head, n, dev_base + off, shape[0], shape[1]),
                             f"rwkvb_packed_init({name})")
                self.descs[name] = DevicePacked(name, d, shape, codec)
            self.host[li] = img
        self._slot_of = (ctypes.c_int32 * n_layer)(*slot_of)
        self._src = (ctypes.c_void_p * n_layer)(*[self.host[li].data_ptr() if li in self.host else None
                                                    for li in range(n_layer)])
        self._dev = (ctypes.c_void_p * self.n_slots)(*[self.slots.data_ptr() + k * self.layer_bytes
                                                        for k in range(self.n_slots)])
        self.desc = native.StageDesc(self.n_slots, self._slot_of, self._src, self._dev, self.layer_bytes)

    @property
    def host_bytes(self) -> int:
        return sum(int(t.numel()) for t in self.host.values())

    @property
    def device_bytes(self) -> int:
        return int(self.slots.numel())


def plan_residency(layer_bytes: dict[int, int], global_bytes: int, n_layer: int, *, hbm_budget: int | None,
                   n_slots: int = 2, resident_layers: list[int] | None = None) -> list[int]:
    """The layers to stream (ascending).  ``resident_layers`` when given, else
    under ``hbm_budget`` bytes of weights: globals (embedding, head) and the
    device slots first, then as many layers as fit in ``hot_layer_order``."""
    if resident_layers is not None:
        keep = set(int(i) for i in resident_layers)
        return [li for li in range(n_layer) if li not in keep]
    if hbm_budget is None:
        return []
    total = global_bytes + sum(layer_bytes.values())
    if total <= hbm_budget:
        return []
    slot = max(layer_bytes.values())
    room = hbm_budget - global_bytes - min(n_slots, n_layer) * slot
    if room < 0:
        raise ValueError(f"HBM budget {hbm_budget} B is below the globals ({global_bytes} B) plus "
                         f"{n_slots} layer slots ({slot} B each)")
    keep = []
    for li in hot_layer_order(n_layer):
        if layer_bytes[li] <= room:
            keep.append(li)
            room -= layer_bytes[li]
    return [li for li in range(n_layer) if li not in set(keep)]
