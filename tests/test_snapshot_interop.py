"""Recurrent-state snapshot files: this backend's writer and reader
(``rwkv_b200.snapshot``) against the reference engine's ``RWS\\x01`` format.

* CPU: round trip of an RWKV-7-shaped state (fp32 and bf16), rejection of a
  bad magic, a truncated payload and a corrupted checksum.
* Where the reference source tree is present: a file written here is read by
  the reference's ``load_snapshot`` and a file written by the reference's
  ``save_snapshot`` is read here, tensors and ``last_token_id`` identical (a
  child process imports a temporary copy of the reference package).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

from rwkv_b200 import snapshot

REPO = Path(__file__).resolve().parents[1]
REF_ROOT = Path(os.environ.get("RWKV_REF_ROOT", "/root/reference"))


def _state(L=3, C=256, H=4, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(L):
        out += [torch.randn(C, generator=g).to(dtype), torch.randn(H, 64, 64, generator=g).to(dtype),
                torch.randn(C, generator=g).to(dtype)]
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_round_trip(tmp_path, dtype):
    st = _state(dtype=dtype)
    p = snapshot.save_snapshot(tmp_path / "s.rws", st, snapshot.SnapshotMeta(prompt="hi", last_token_id=42))
    got, meta = snapshot.load_snapshot(p)
    assert meta.last_token_id == 42 and meta.prompt == "hi" and meta.backend == "cuda_b200"
    assert len(got) == len(st)
    for a, b in zip(st, got):
        assert a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)


def test_rejects_bad_files(tmp_path):
    p = snapshot.save_snapshot(tmp_path / "s.rws", _state(), snapshot.SnapshotMeta(last_token_id=1))
    raw = bytearray(p.read_bytes())
    bad = tmp_path / "bad.rws"
    bad.write_bytes(b"XXXX" + bytes(raw[4:]))
    with pytest.raises(ValueError, match="magic"):
        snapshot.load_snapshot(bad)
    bad.write_bytes(bytes(raw[: len(raw) // 2]))
    with pytest.raises(ValueError):
        snapshot.load_snapshot(bad)
    flipped = bytearray(raw)
    flipped[len(flipped) // 2] ^= 0xFF
    bad.write_bytes(bytes(flipped))
    with pytest.raises(ValueError, match="checksum"):
        snapshot.load_snapshot(bad)


_CROSS = textwrap.dedent('''
    import sys, torch
    from pathlib import Path
    from rwkv_ssd.runtime import snapshot as ref
    from rwkv_ssd.runtime.state_cache import RecurrentState
    from rwkv_b200 import snapshot as ours
    d = Path(sys.argv[1])
    g = torch.Generator().manual_seed(5)
    st = []
    for _ in range(2):
        st += [torch.randn(256, generator=g), torch.randn(4, 64, 64, generator=g), torch.randn(256, generator=g)]
    # ours -> reference
    ours.save_snapshot(d / "ours.rws", st, ours.SnapshotMeta(prompt="p", last_token_id=77))
    rs, rm = ref.load_snapshot(d / "ours.rws")
    assert rm.last_token_id == 77 and rm.backend == "cuda_b200" and rs.last_token_id == 77
    assert rs.h is None and len(rs.rwkv7_state) == len(st)
    assert all(torch.equal(a, b) for a, b in zip(st, rs.rwkv7_state))
    # reference -> ours
    ref.save_snapshot(d / "ref.rws", RecurrentState(last_token_id=9, rwkv7_state=st),
                      ref.SnapshotMeta(backend="chatrwkv", mode="resident", model_family="rwkv7", last_token_id=9))
    os_, om = ours.load_snapshot(d / "ref.rws")
    assert om.last_token_id == 9 and om.backend == "chatrwkv"
    assert all(torch.equal(a, b) for a, b in zip(st, os_))
    print("cross ok")
''')


@pytest.mark.skipif(not (REF_ROOT / "rwkv_ssd" / "runtime" / "snapshot.py").is_file(),
                    reason="reference source tree not present")
def test_files_cross_read_with_the_reference(tmp_path):
    shutil.copytree(REF_ROOT / "rwkv_ssd", tmp_path / "rwkv_ssd",
                    ignore=shutil.ignore_patterns("*.dll", "__pycache__", "*.so"))
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(tmp_path), str(REPO / "ssd-rwkv-engine_b200"), str(REPO)])
    r = subprocess.run([sys.executable, "-c", _CROSS, str(tmp_path)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "cross ok" in r.stdout
