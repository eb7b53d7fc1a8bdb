"""Residency tiers on the GPU: layers streamed from pinned host memory through
device slots (``rwkvb_engine_create_staged``) decode exactly as the fully
resident engine.

The staged engine runs the same multi-kernel step on the same bytes, so its
logits must be bit-identical to the resident multi-kernel engine's, for every
slot count, with and without the CUDA graph; and the plugin's ``partial`` /
``streaming`` modes and HBM budget give the oracle's greedy ids."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle.forward import OracleRWKV7  # noqa: E402
from rwkv_b200 import backend as bk  # noqa: E402
from rwkv_b200 import synth  # noqa: E402
from rwkv_b200.engine import B200BatchEngine, B200Engine, ModelUpload  # noqa: E402

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def tiny():
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 41, "cpu"), policy="sg8")
    prompt = synth.seeded_prompt(6, shape.vocab, 41)
    ref = B200Engine(pack, persistent=False)
    rows = []
    for t in prompt:
        ref.forward([t])
        rows.append(ref.logits.clone())
    ids = ref.decode_greedy(int(torch.argmax(ref.logits)), 8)
    state = [t.clone() for t in ref.get_state()]
    ref.close()
    return shape, pack, prompt, torch.stack(rows), ids, state


@pytest.mark.parametrize("resident,slots,graph", [([0], 2, True), ([], 2, True), ([1, 2], 1, True),
                                                  ([0, 3], 3, False)])
def test_staged_layers_are_bit_identical_to_resident(tiny, resident, slots, graph):
    shape, pack, prompt, rows_ref, ids_ref, state_ref = tiny
    up = ModelUpload(pack, DEV, resident_layers=resident, stage_slots=slots)
    assert up.stage is not None and up.stage.streamed == [i for i in range(shape.n_layer) if i not in resident]
    assert up.stage.n_slots == min(slots, len(up.stage.streamed))
    eng = B200Engine(up, use_graph=graph)
    try:
        assert not eng.persistent_active
        rows = []
        for t in prompt:
            eng.forward([t])
            rows.append(eng.logits.clone())
        assert torch.equal(torch.stack(rows), rows_ref)
        assert eng.decode_greedy(int(torch.argmax(eng.logits)), 8) == ids_ref
        for a, b in zip(eng.get_state(), state_ref):
            assert torch.equal(a, b)
    finally:
        eng.close()


def test_budget_keeps_hot_layers_and_streams_the_rest(tiny):
    shape, pack, prompt, rows_ref, ids_ref, _ = tiny
    full = ModelUpload(pack, DEV)
    assert full.stage is None
    layer = ModelUpload(pack, DEV, resident_layers=[]).stage.layer_bytes
    budget = full.weights.nbytes - layer // 2  # half a layer short of the whole model
    del full
    up = ModelUpload(pack, DEV, hbm_budget=budget, stage_slots=2)
    assert up.stage is not None and 0 < len(up.stage.streamed) < shape.n_layer
    assert up.weights.nbytes + up.stage.device_bytes <= budget
    assert 0 not in up.stage.streamed  # the outermost layers are the hot ones
    eng = B200Engine(up)
    try:
        eng.forward(prompt)
        assert torch.equal(eng.logits, rows_ref[-1])
        assert eng.decode_greedy(int(torch.argmax(eng.logits)), 8) == ids_ref
    finally:
        eng.close()
    with pytest.raises(ValueError):
        B200BatchEngine(up, 2)  # the batched engine needs every layer resident


@pytest.mark.parametrize("mode", ["partial", "streaming"])
def test_plugin_residency_modes_match_oracle(mode):
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 43, "cpu"), policy="sg8")
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    b = bk.create_backend("cuda_b200")
    b.load_pack(None, "cuda:0")
    b.prepare_provider(bk.PackProvider(pack), config=types.SimpleNamespace(mode=mode, residency_profile=None))
    try:
        streamed = b._model.stage.streamed
        assert streamed == ([1, 2] if mode == "partial" else [0, 1, 2, 3])
        prompt = synth.seeded_prompt(5, shape.vocab, 43)
        st = b.prefill_tokens(prompt)
        ids = b.decode_greedy(st, None, 6, metrics=None)
        ref_ids, ref_logits, _ = oracle.greedy(prompt, 6)
        assert ids == ref_ids
        np.testing.assert_allclose(b.probe_logits(st).cpu().numpy(), ref_logits[len(prompt) - 1], atol=1e-3, rtol=0)
        assert b.capabilities()["declared"]["pack_streaming"]
    finally:
        b.close()
