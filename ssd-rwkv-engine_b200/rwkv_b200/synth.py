"""Seeded RWKV-7 models and pack encoders for synthetic workloads.

No checkpoints are available to this engine's benchmarks, so every model is
a seeded random RWKV-7 state dict with the reference checkpoint's tensor
names and shapes, packed with the reference codecs:

* ``SG8\\x01`` grouped affine UINT8 — ``encode_sg8`` restates
  ``encode_scale_u8_grouped`` (reference ``rwkv_ssd/runtime/pack_codec.py:33-68``)
  in torch, so that multi-GB packs can be encoded on the GPU.  Its bytes are
  identical to the reference encoder's on the same fp32 input (pinned by the
  CPU tests).
* ``TR2\\x04`` grouped LUT2 (2-bit codes, 4-entry fp16 codebook per group) —
  ``encode_lut2`` follows ``encode_trinity_lut2(codebook="groupwise_kmeans_fp16")``
  (reference ``rwkv_ssd/runtime/trinity_codec.py:494-623``,
  ``trinity_codebook.py:139-195``) in torch.  It is used to *generate* large
  benchmark packs; parity tests use packs made by the reference encoder.

Codec policies mirror the reference packer (``rwkv_ssd/tools/pack_runtime.py``):
``"sg8"`` is the ``native_safe`` preset (every 2-D tensor grouped-U8, others
lossless, ``pack_runtime.py:300-327``); ``"lut2"`` keeps the large projections
(att r/k/v/o, ffn key/value, head) in ``TR2\\x04`` and the remaining 2-D
tensors in grouped-U8, as a ``legacy`` preset with a ``codec_map`` would.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np
import torch

SG8_MAGIC = b"SG8\x01"
LUT2_FP16_MAGIC = b"TR2\x04"


@dataclass(frozen=True)
class RWKV7Shape:
    """Dimensions of an RWKV-7 model (``x070`` layout)."""

    n_layer: int
    n_embd: int
    head_size: int
    ffn: int
    vocab: int
    rank_w: int
    rank_a: int
    rank_v: int
    rank_g: int

    @property
    def n_head(self) -> int:
        return self.n_embd // self.head_size

    def weights_per_token(self) -> int:
        """Packed matrix elements read per decoded token (embedding row excluded)."""
        C, F = self.n_embd, self.ffn
        per_layer = 4 * C * C + 2 * C * F + 2 * C * (self.rank_w + self.rank_a + self.rank_g)
        per_layer_v = 2 * C * self.rank_v
        return self.n_layer * per_layer + (self.n_layer - 1) * per_layer_v + self.vocab * C


# Shapes of the reference benchmark configurations (LoRA ranks follow the
# public RWKV-7 rank rule for each width).
PRESETS: dict[str, RWKV7Shape] = {
    "tiny": RWKV7Shape(4, 256, 64, 1024, 1024, 32, 32, 32, 64),
    "0.1b": RWKV7Shape(12, 768, 64, 3072, 65536, 64, 64, 32, 128),
    "2.9b": RWKV7Shape(32, 2560, 64, 10240, 65536, 96, 96, 64, 320),
    "7.2b": RWKV7Shape(32, 4096, 64, 16384, 65536, 128, 128, 96, 480),
    # 2.9B widths with 4 layers: per-kernel profiling case (~0.5 GB, larger than L2)
    "2.9b-l4": RWKV7Shape(4, 2560, 64, 10240, 65536, 96, 96, 64, 320),
    "7.2b-l4": RWKV7Shape(4, 4096, 64, 16384, 65536, 128, 128, 96, 480),
}


def tensor_specs(s: RWKV7Shape) -> list[tuple[str, tuple[int, ...], str]]:
    """``(name, checkpoint shape, init kind)`` in checkpoint order."""
    C, H, N, F, V = s.n_embd, s.n_head, s.head_size, s.ffn, s.vocab
    out: list[tuple[str, tuple[int, ...], str]] = [("emb.weight", (V, C), "normal")]
    for i in range(s.n_layer):
        b = f"blocks.{i}."
        if i == 0:
            out += [(b + "ln0.weight", (C,), "ln_w"), (b + "ln0.bias", (C,), "ln_b")]
        out += [(b + "ln1.weight", (C,), "ln_w"), (b + "ln1.bias", (C,), "ln_b"),
                (b + "ln2.weight", (C,), "ln_w"), (b + "ln2.bias", (C,), "ln_b")]
        a = b + "att."
        for nm in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
            out.append((a + nm, (1, 1, C), "unit"))
        out += [(a + "w0", (1, 1, C), "decay0"), (a + "w1", (C, s.rank_w), "normal"),
                (a + "w2", (s.rank_w, C), "normal"),
                (a + "a0", (1, 1, C), "sym"), (a + "a1", (C, s.rank_a), "normal"),
                (a + "a2", (s.rank_a, C), "normal")]
        # Layer 0 carries v0/v1/v2 in the checkpoint although its TMix never
        # reads them (it defines v_first instead).
        out += [(a + "v0", (1, 1, C), "sym"), (a + "v1", (C, s.rank_v), "normal"),
                (a + "v2", (s.rank_v, C), "normal")]
        out += [(a + "g1", (C, s.rank_g), "normal"), (a + "g2", (s.rank_g, C), "normal"),
                (a + "k_k", (1, 1, C), "around1"), (a + "k_a", (1, 1, C), "around1"),
                (a + "r_k", (H, N), "rk"),
                (a + "receptance.weight", (C, C), "normal"), (a + "key.weight", (C, C), "normal"),
                (a + "value.weight", (C, C), "normal"), (a + "output.weight", (C, C), "normal"),
                (a + "ln_x.weight", (C,), "ln_w"), (a + "ln_x.bias", (C,), "ln_b")]
        f = b + "ffn."
        out += [(f + "x_k", (1, 1, C), "unit"), (f + "key.weight", (F, C), "normal"),
                (f + "value.weight", (C, F), "normal")]
    out += [("ln_out.weight", (C,), "ln_w"), ("ln_out.bias", (C,), "ln_b"),
            ("head.weight", (V, C), "normal")]
    return out


def _draw(kind: str, shape: tuple[int, ...], gen: torch.Generator, device) -> torch.Tensor:
    kw = dict(generator=gen, device=device, dtype=torch.float32)
    if kind == "normal":
        return torch.randn(shape, **kw) * 0.02
    u = torch.rand(shape, **kw)
    if kind == "unit":
        return u
    if kind == "ln_w":
        return 1.0 + 0.2 * (u - 0.5)
    if kind == "ln_b":
        return 0.2 * (u - 0.5)
    if kind == "decay0":
        return 4.0 * u - 3.0
    if kind == "sym":
        return 2.0 * u - 1.0
    if kind == "around1":
        return 0.5 + u
    if kind == "rk":
        return (u - 0.5) * 0.4
    raise ValueError(kind)


def generate_state_dict(s: RWKV7Shape, seed: int, device="cpu") -> dict[str, torch.Tensor]:
    """Seeded fp32 RWKV-7 state dict.

    Matrices ~ N(0, 0.02); token-shift mixes ~ U(0, 1); norms 1±0.1 / ±0.1;
    ``w0`` ~ U(-3, 1); ``a0``/``v0`` ~ U(-1, 1); ``k_k``/``k_a`` ~ U(0.5, 1.5);
    ``r_k`` ~ U(-0.2, 0.2).  Draws use one ``torch.Generator`` seeded with
    ``seed`` on ``device`` in checkpoint order (CPU and CUDA streams differ).
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    return {n: _draw(k, shp, gen, device) for n, shp, k in tensor_specs(s)}


# --------------------------------------------------------------------------
# encoders (torch; CPU or CUDA)
# --------------------------------------------------------------------------
def encode_sg8(t: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """SG8 blob bytes as a uint8 tensor on ``t.device``.

    Same arithmetic as ``encode_scale_u8_grouped``: per-group fp32 min/max
    (degenerate range -> max = min + 1), ``rint((w - min) / (max - min) * 255)``
    clipped to [0, 255]; the partial last group is padded with its last value.
    """
    flat = t.detach().to(torch.float32).reshape(-1)
    n = flat.numel()
    g = int(group_size)
    groups = (n + g - 1) // g
    scales = torch.empty((groups, 2), dtype=torch.float32, device=flat.device)
    quant = torch.empty(n, dtype=torch.uint8, device=flat.device)
    step = max(1, (1 << 26) // g)
    for first in range(0, groups, step):
        cnt = min(step, groups - first)
        start = first * g
        avail = min(cnt * g, n - start)
        chunk = flat[start:start + avail]
        if avail < cnt * g:
            chunk = torch.cat([chunk, chunk[-1:].expand(cnt * g - avail)])
        chunk = chunk.reshape(cnt, g)
        lo = chunk.amin(dim=1)
        hi = chunk.amax(dim=1)
        hi = torch.where(hi - lo < 1e-12, lo + 1.0, hi)
        scales[first:first + cnt, 0] = lo
        scales[first:first + cnt, 1] = hi
        q = torch.round((chunk - lo[:, None]) / (hi - lo)[:, None] * 255.0).clamp_(0, 255)
        quant[start:start + avail] = q.reshape(-1)[:avail].to(torch.uint8)
    head = torch.frombuffer(bytearray(SG8_MAGIC + struct.pack("<I", g)), dtype=torch.uint8)
    return torch.cat([head.to(flat.device), scales.reshape(-1).view(torch.uint8), quant])


def _pack_2bit_t(idx: torch.Tensor) -> torch.Tensor:
    n = idx.numel()
    pad = (4 - n % 4) % 4
    if pad:
        idx = torch.cat([idx, torch.zeros(pad, dtype=idx.dtype, device=idx.device)])
    v = idx.to(torch.uint8).reshape(-1, 4)
    return v[:, 0] | (v[:, 1] << 2) | (v[:, 2] << 4) | (v[:, 3] << 6)


def encode_lut2(t: torch.Tensor, group_size: int = 64, iters: int = 12) -> torch.Tensor:
    """``TR2\\x04`` blob bytes as a uint8 tensor on ``t.device``.

    Per contiguous group: quantile-initialised 1-D k-means with four sorted
    centroids, rounded to fp16; codes = nearest centroid (first on ties).
    """
    flat = t.detach().to(torch.float32).reshape(-1)
    n = flat.numel()
    g = int(group_size)
    groups = (n + g - 1) // g
    cbs = torch.empty((groups, 4), dtype=torch.float16, device=flat.device)
    codes = torch.empty(n, dtype=torch.uint8, device=flat.device)
    q = torch.tensor([0.2, 0.4, 0.6, 0.8], dtype=torch.float32, device=flat.device)
    step = max(1, (1 << 24) // g)
    for first in range(0, groups, step):
        cnt = min(step, groups - first)
        start = first * g
        avail = min(cnt * g, n - start)
        chunk = flat[start:start + avail]
        if avail < cnt * g:
            chunk = torch.cat([chunk, chunk[-1:].expand(cnt * g - avail)])
        chunk = chunk.reshape(cnt, g)
        valid = (torch.arange(cnt * g, device=flat.device) < avail).reshape(cnt, g)
        centers = torch.quantile(chunk, q, dim=1).T.contiguous()
        for _ in range(max(1, iters)):
            lab = (chunk[:, :, None] - centers[:, None, :]).abs().argmin(dim=2)
            oh = torch.nn.functional.one_hot(lab, 4).to(torch.float64) * valid[:, :, None]
            cnts = oh.sum(dim=1)
            sums = (oh * chunk.to(torch.float64)[:, :, None]).sum(dim=1)
            upd = torch.where(cnts > 0, (sums / cnts.clamp_min(1)).to(torch.float32), centers)
            upd, _ = upd.sort(dim=1)
            done = (upd - centers).abs().max() < 1e-7
            centers = upd
            if bool(done):
                break
        c16 = centers.to(torch.float16)
        cbs[first:first + cnt] = c16
        lab = (chunk[:, :, None] - c16.to(torch.float32)[:, None, :]).abs().argmin(dim=2)
        codes[start:start + avail] = lab.reshape(-1)[:avail].to(torch.uint8)
    head = torch.frombuffer(bytearray(LUT2_FP16_MAGIC + struct.pack("<I", g)), dtype=torch.uint8)
    return torch.cat([head.to(flat.device), cbs.reshape(-1).view(torch.uint8), _pack_2bit_t(codes)])


# --------------------------------------------------------------------------
# packs
# --------------------------------------------------------------------------
@dataclass
class PackedTensor:
    """One pack entry: ``codec`` is ``"sg8"``, ``"lut2"`` or ``"none"``;
    ``payload`` is the wire blob (bytes or a uint8 tensor) or, for
    ``"none"``, the fp32 values."""

    name: str
    shape: tuple[int, ...]
    codec: str
    payload: object
    meta: dict = field(default_factory=dict)


_LUT2_SUFFIXES = (".att.receptance.weight", ".att.key.weight", ".att.value.weight",
                  ".att.output.weight", ".ffn.key.weight", ".ffn.value.weight")


def codec_for(name: str, shape: tuple[int, ...], policy: str) -> str:
    if len(shape) != 2:
        return "none"
    if policy == "lut2" and (name == "head.weight" or name.endswith(_LUT2_SUFFIXES)):
        return "lut2"
    return "sg8"


def make_pack(sd: dict[str, torch.Tensor], *, policy: str = "sg8", sg8_group: int = 128,
              lut2_group: int = 64, as_bytes: bool = True) -> dict[str, PackedTensor]:
    """Encode a state dict.  ``as_bytes`` returns host ``bytes`` payloads;
    otherwise blobs stay uint8 tensors on the state dict's device."""
    out: dict[str, PackedTensor] = {}
    for name, t in sd.items():
        shape = tuple(int(d) for d in t.shape)
        codec = codec_for(name, shape, policy)
        if codec == "sg8":
            blob = encode_sg8(t, sg8_group)
        elif codec == "lut2":
            blob = encode_lut2(t, lut2_group)
        else:
            v = t.detach().to(torch.float32).reshape(-1)
            out[name] = PackedTensor(name, shape, "none",
                                     v.cpu().numpy().copy() if as_bytes else v)
            continue
        out[name] = PackedTensor(name, shape, codec, blob.cpu().numpy().tobytes() if as_bytes else blob)
    return out


def seeded_prompt(n: int, vocab: int, seed: int) -> list[int]:
    """``n`` token ids ~ U[0, vocab) from a seeded CPU generator."""
    gen = torch.Generator().manual_seed(int(seed) + 7919)
    return [int(v) for v in torch.randint(0, vocab, (n,), generator=gen)]


def packed_nbytes(pack: dict[str, PackedTensor], names=None) -> int:
    tot = 0
    for n, e in pack.items():
        if names is not None and n not in names:
            continue
        p = e.payload
        tot += len(p) if isinstance(p, (bytes, bytearray)) else int(np.prod(getattr(p, "shape", (0,)))) * (
            1 if e.codec != "none" else 4)
    return tot


def make_pack_streaming(s: RWKV7Shape, seed: int, device="cuda", *, policy: str = "sg8", sg8_group: int = 128,
                        lut2_group: int = 64, transform=None) -> dict[str, PackedTensor]:
    """Draw and encode one tensor at a time on ``device`` (blobs stay uint8
    tensors there), so multi-GB packs never hold the whole fp32 model.
    ``transform(name, entry) -> entry``, when given, is applied to each entry as
    it is made (e.g. keeping one tensor-parallel shard of it)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    out: dict[str, PackedTensor] = {}
    for name, shp, kind in tensor_specs(s):
        t = _draw(kind, shp, gen, device)
        codec = codec_for(name, shp, policy)
        if codec == "sg8":
            payload = encode_sg8(t, sg8_group)
        elif codec == "lut2":
            payload = encode_lut2(t, lut2_group)
        else:
            payload = t.reshape(-1).clone()
        entry = PackedTensor(name, shp, codec, payload)
        out[name] = transform(name, entry) if transform is not None else entry
        del t, payload, entry
    return out


def pack_to_host(pack: dict[str, PackedTensor]) -> dict[str, PackedTensor]:
    """Host copy (bytes / fp32 numpy) of a device-resident pack."""
    out = {}
    for n, e in pack.items():
        p = e.payload
        if isinstance(p, torch.Tensor):
            p = p.cpu().numpy()
            p = p.tobytes() if e.codec != "none" else p.astype(np.float32)
        out[n] = PackedTensor(n, e.shape, e.codec, p)
    return out
