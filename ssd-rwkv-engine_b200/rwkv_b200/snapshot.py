"""Recurrent-state snapshot files in the reference engine's format.

The file is the reference's ``RWS\\x01`` snapshot (``rwkv_ssd/runtime/snapshot.py:
261-306``) so that states move between this backend and the reference engine in
either direction:

* magic ``b"RWS\\x01"``;
* ``u32`` little-endian header length, then a JSON header (``sort_keys``) with
  ``version`` 2, ``specs`` (shape, dtype code, byte count per tensor),
  ``state_kind`` (``"rwkv7"`` here) and the ``meta`` dictionary;
* the tensors' raw little-endian bytes back to back (fp32 dtype code 2, bf16
  1, fp16 3, int32 4);
* a trailer: ``u64`` payload size and the payload's sha256 as 64 hex characters.

A snapshot carries the *portable* state form: ``rwkv7_state`` is the state
before ``last_token_id`` was consumed (per layer ``[x_prev_att, S, x_prev_ffn]``),
and a reader resumes by consuming ``last_token_id`` first, as the reference's
``decode_greedy_from_state`` (``rwkv7_forward.py:941-990``) does.
"""

from __future__ import annotations

import hashlib
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import torch

MAGIC = b"RWS\x01"
VERSION = 2
_CODES = {torch.bfloat16: 1, torch.float32: 2, torch.float16: 3, torch.int32: 4}
_DTYPES = {v: k for k, v in _CODES.items()}


@dataclass
class SnapshotMeta:
    """Field-compatible with the reference ``SnapshotMeta`` (snapshot.py:118-161)."""

    backend: str = "cuda_b200"
    mode: str = "resident"
    model_family: str = "rwkv7"
    max_layers_in_z: int = 1
    decouple_provider_cache: bool = True
    max_provider_cache_layers: int = 0
    prompt: str = ""
    last_token_id: int = 0
    extras: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = {"backend": self.backend, "mode": self.mode, "model_family": self.model_family,
             "max_layers_in_z": self.max_layers_in_z, "decouple_provider_cache": self.decouple_provider_cache,
             "max_provider_cache_layers": self.max_provider_cache_layers, "prompt": self.prompt,
             "last_token_id": self.last_token_id}
        if self.extras:
            d["extras"] = dict(self.extras)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "SnapshotMeta":
        return cls(backend=str(d.get("backend", "cuda_b200")), mode=str(d.get("mode", "resident")),
                   model_family=str(d.get("model_family", "rwkv7")),
                   max_layers_in_z=int(d.get("max_layers_in_z", 1)),
                   decouple_provider_cache=bool(d.get("decouple_provider_cache", True)),
                   max_provider_cache_layers=int(d.get("max_provider_cache_layers", 0)),
                   prompt=str(d.get("prompt", "")), last_token_id=int(d.get("last_token_id", 0)),
                   extras=dict(d.get("extras", {}) or {}))


def _tensor_bytes(t: torch.Tensor) -> bytes:
    c = t.detach().contiguous().cpu()
    if c.dtype == torch.bfloat16:
        return c.view(torch.uint16).numpy().tobytes()
    return c.numpy().tobytes()


def save_snapshot(path, rwkv7_state: list[torch.Tensor], meta: SnapshotMeta) -> Path:
    """Write ``rwkv7_state`` (portable form: the state before
    ``meta.last_token_id``) and ``meta`` to ``path`` (via a ``.tmp`` file)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    specs, parts = [], []
    for t in rwkv7_state:
        if t.dtype not in _CODES:
            raise ValueError(f"unsupported state dtype {t.dtype}")
        b = _tensor_bytes(t)
        specs.append({"shape": list(t.shape), "dtype_code": _CODES[t.dtype], "nbytes": len(b)})
        parts.append(b)
    payload = b"".join(parts)
    header = {"version": VERSION, "specs": specs, "state_kind": "rwkv7", "meta": meta.to_dict()}
    hb = json.dumps(header, sort_keys=True).encode("utf-8")
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("wb") as fh:
        fh.write(MAGIC)
        fh.write(struct.pack("<I", len(hb)))
        fh.write(hb)
        fh.write(payload)
        fh.write(struct.pack("<Q", len(payload)))
        fh.write(hashlib.sha256(payload).hexdigest().encode("ascii"))
    tmp.replace(path)
    return path


def load_snapshot(path) -> tuple[list[torch.Tensor], SnapshotMeta]:
    """Read a snapshot written by this module or by the reference engine;
    returns the ``rwkv7_state`` tensors (host) and the metadata.  Raises
    ``ValueError`` on a bad magic, version, truncation, size or checksum, or a
    snapshot that holds no RWKV-7 state."""
    path = Path(path)
    with path.open("rb") as fh:
        if fh.read(4) != MAGIC:
            raise ValueError(f"bad snapshot magic in {path}")
        (hl,) = struct.unpack("<I", fh.read(4))
        header = json.loads(fh.read(hl).decode("utf-8"))
        if int(header.get("version", 0)) not in (1, VERSION):
            raise ValueError(f"unsupported snapshot version {header.get('version')}")
        specs = header.get("specs") or []
        total = sum(int(s["nbytes"]) for s in specs)
        ext = header.get("external_spec") or None
        total += int(ext.get("nbytes", 0)) if ext else 0
        payload = fh.read(total)
        if len(payload) != total:
            raise ValueError(f"snapshot payload truncated in {path}")
        tail = fh.read(8)
        if len(tail) != 8 or struct.unpack("<Q", tail)[0] != total:
            raise ValueError(f"snapshot payload size mismatch in {path}")
        sha = fh.read(64).decode("ascii", errors="replace")
        if sha and hashlib.sha256(payload).hexdigest() != sha:
            raise ValueError(f"snapshot payload checksum mismatch in {path}")
    meta = SnapshotMeta.from_dict(header.get("meta") or {})
    kind = header.get("state_kind") or ("rwkv7" if len(specs) != 1 else "h")
    if kind != "rwkv7":
        raise ValueError(f"snapshot holds a {kind!r} state, not an RWKV-7 state")
    out, cur = [], 0
    for s in specs:
        n = int(s["nbytes"])
        dt = _DTYPES[int(s["dtype_code"])]
        raw = bytearray(payload[cur:cur + n])
        if dt == torch.bfloat16:
            t = torch.frombuffer(raw, dtype=torch.int16).view(torch.bfloat16)
        else:
            t = torch.frombuffer(raw, dtype=dt)
        out.append(t.reshape(list(s["shape"])).clone())
        cur += n
    return out, meta
