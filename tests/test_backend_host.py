"""Host-side behaviour of the ``cuda_b200`` backend plugin (no GPU needed).

Mirrors the reference's backend tests in spirit: provider fakes built with
``SimpleNamespace`` (reference ``tests/test_fused_lut_forward.py:20-193``),
factory keys (``backends/factory.py:32-78``) and generation control
(``runtime/generation_control.py``).
"""

from __future__ import annotations

import threading
import time
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from rwkv_b200 import backend as bk
from rwkv_b200 import synth


def _manifest_provider(pack: dict) -> SimpleNamespace:
    """A reference-style provider: ``manifest.tensors`` + ``_read_packed_bytes``."""
    entries, blobs = [], {}
    for name, e in pack.items():
        if e.codec == "none":
            raw = np.asarray(e.payload, np.float32).tobytes()
            dq = "none"
        else:
            raw = e.payload
            dq = "scale_u8_grouped" if e.codec == "sg8" else "trinity_lut2"
        entries.append(SimpleNamespace(name=name, shape=list(e.shape), dtype="float32", dequant=dq, layer_id=0))
        blobs[name] = raw
    return SimpleNamespace(manifest=SimpleNamespace(tensors=entries),
                           _read_packed_bytes=lambda entry, timing: blobs[entry.name])


def test_factory_keys_and_errors():
    assert isinstance(bk.create_backend("cuda_b200"), bk.CudaB200Backend)
    assert isinstance(bk.create_backend(" B200 "), bk.CudaB200Backend)
    with pytest.raises(ValueError):
        bk.create_backend("rwkvcpp")
    with pytest.raises(ValueError):
        bk.ensure_v0_backend("nope")
    if not torch.cuda.is_available():
        with pytest.raises(bk.BackendNotAvailableError):
            bk.ensure_v0_backend("cuda_b200")


def test_provider_conversion_matches_pack():
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 5, "cpu"), policy="sg8")
    got = bk.packed_tensors_from_provider(_manifest_provider(pack))
    assert set(got) == set(pack)
    for n, e in pack.items():
        assert got[n].codec == e.codec
        if e.codec == "none":
            np.testing.assert_array_equal(got[n].payload, np.asarray(e.payload, np.float32))
        else:
            assert got[n].payload == e.payload


def test_provider_conversion_decodes_bf16_vectors_and_rejects_unknown_codecs():
    vals = torch.tensor([1.5, -2.25, 0.0078125], dtype=torch.bfloat16)
    raw = vals.view(torch.uint16).numpy().tobytes()
    prov = SimpleNamespace(
        manifest=SimpleNamespace(tensors=[SimpleNamespace(name="v", shape=[3], dtype="bfloat16", dequant="none")]),
        _read_packed_bytes=lambda e, t: raw)
    got = bk.packed_tensors_from_provider(prov)["v"]
    np.testing.assert_array_equal(got.payload, vals.float().numpy())
    bad = SimpleNamespace(
        manifest=SimpleNamespace(tensors=[SimpleNamespace(name="w", shape=[4, 4], dtype="float32", dequant="scale_u4")]),
        _read_packed_bytes=lambda e, t: b"\0" * 16)
    with pytest.raises(bk.CapabilityNotSupportedError):
        bk.packed_tensors_from_provider(bad)
    with pytest.raises(TypeError):
        bk.packed_tensors_from_provider(object())


def test_pack_provider_fused_blob_protocol():
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 5, "cpu"), policy="sg8")
    prov = bk.PackProvider(pack)
    blob, out_f, in_f = prov.get_fused_lut_blob("blocks.0.att.key.weight")
    assert (out_f, in_f) == (256, 256) and bytes(blob[:4]) == b"SG8\x01"
    assert prov.get_fused_lut_blob("blocks.0.att.x_r") is None
    assert prov._use_fused_lut_matmul()


def test_recurrent_state_clone_is_deep():
    st = bk.RecurrentState(3, None, [torch.zeros(2), torch.ones(1, 2, 2), torch.zeros(2)],
                           {"pending_logits": torch.arange(4.0)})
    cl = st.clone()
    cl.rwkv7_state[1] += 1
    cl.external_state["pending_logits"][0] = 9
    assert float(st.rwkv7_state[1].sum()) == 4.0
    assert float(st.external_state["pending_logits"][0]) == 0.0


def test_generation_control_cancel_deadline_callback():
    seen = []
    ctl = bk._control(token_callback=seen.append)
    ctl.emit(7)
    assert seen == [7]
    ev = threading.Event()
    ev.set()
    with pytest.raises(bk.GenerationCancelled):
        bk._control(cancel_event=ev).check()
    with pytest.raises(bk.GenerationCancelled):
        bk._control(deadline=time.monotonic() - 1).check()
    assert bk._control() is None


def test_capabilities_and_unloaded_errors():
    b = bk.CudaB200Backend()
    caps = b.capabilities()
    assert caps["name"] == "cuda_b200"
    assert "scale_u8_grouped" in caps["declared"]["supported_codecs"]
    assert b.supports_capability("logits_probe")
    # no prefix cache is built: the backend must not claim one
    assert not b.supports_capability("prefix_cache")
    assert b.get_recurrent_state() is None and b.probe_logits() is None
    with pytest.raises(RuntimeError):
        b._engine_or_raise()
    with pytest.raises(bk.CapabilityNotSupportedError):
        b.load("x.pth", "cuda fp32", "cuda")
    with pytest.raises(bk.CapabilityNotSupportedError):
        b._encode("hello")
    with pytest.raises(bk.BackendNotAvailableError):
        b.load_pack(SimpleNamespace(tensors=[]), "cpu")
