"""GPU parity of the batched decode engine (``rwkvb_batch_*``): every session of
a batch must decode exactly as the reference's per-session loop (the oracle
forward, pinned to the reference's ``forward_block_packed``) and as the batch-1
engine: greedy ids identical, logits and recurrent state within 1e-3 max-abs
(the contract allows 1e-2)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle.forward import OracleRWKV7  # noqa: E402
from rwkv_b200 import synth  # noqa: E402
from rwkv_b200.engine import B200BatchEngine, B200Engine  # noqa: E402
from rwkv_b200.native import RwkvbError  # noqa: E402

TOL = 1e-3


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _pack(preset: str, seed: int):
    shape = synth.PRESETS[preset]
    return shape, synth.make_pack(synth.generate_state_dict(shape, seed, "cpu"), policy="sg8")


def _prompts(n: int, length: int, vocab: int, seed: int) -> list[list[int]]:
    return [synth.seeded_prompt(length, vocab, seed + 101 * b) for b in range(n)]


def _prefill(eng: B200BatchEngine, prompts: list[list[int]]) -> None:
    for pos in range(len(prompts[0])):
        eng.forward([p[pos] for p in prompts])


@pytest.mark.parametrize("use_graph", [True, False])
def test_batch_sessions_match_oracle(use_graph):
    shape, pack = _pack("tiny", 7)
    nb, n_new = 5, 12
    prompts = _prompts(nb, 8, shape.vocab, 7)
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    eng = B200BatchEngine(pack, nb, use_graph=use_graph)
    try:
        _prefill(eng, prompts)
        first = _np(eng.logits).argmax(axis=1)
        ids = eng.decode_greedy(n_new)
        logits = _np(eng.logits)
        for b in range(nb):
            ids_ref, logits_ref, state_ref = oracle.greedy(prompts[b], n_new + 1)
            assert int(first[b]) == ids_ref[0]
            assert [int(t) for t in ids[:, b]] == ids_ref[1:], b
            np.testing.assert_allclose(logits[b], logits_ref[-1], rtol=0, atol=TOL)
            st = eng.get_state(b)
            for j, s in enumerate(st):
                np.testing.assert_allclose(_np(s).reshape(-1), state_ref[j].reshape(-1), rtol=0, atol=TOL)
    finally:
        eng.close()


def test_batch_graph_and_plain_launches_agree_bitwise():
    shape, pack = _pack("tiny", 9)
    prompts = _prompts(3, 4, shape.vocab, 9)
    out = []
    for use_graph in (True, False):
        eng = B200BatchEngine(pack, 3, use_graph=use_graph)
        try:
            _prefill(eng, prompts)
            ids = eng.decode_greedy(6)
            out.append((ids, eng.logits.clone(), eng.wkv.clone()))
        finally:
            eng.close()
    assert np.array_equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])
    assert torch.equal(out[0][2], out[1][2])


@pytest.mark.parametrize("preset,nb,steps", [("0.1b", 64, 4), ("2.9b-l4", 64, 3)])
def test_batch_matches_batch1_engine(preset, nb, steps):
    """Full-width shapes at batch 64: sessions 0, 17 and nb-1 against the batch-1 engine."""
    shape = synth.PRESETS[preset]
    pack = synth.make_pack_streaming(shape, 5, "cuda", policy="sg8")
    prompts = _prompts(nb, 3, shape.vocab, 5)
    eng = B200BatchEngine(pack, nb)
    one = B200Engine(pack)
    try:
        _prefill(eng, prompts)
        ids = eng.decode_greedy(steps)
        logits = _np(eng.logits)
        for b in (0, 17, nb - 1):
            one.reset()
            ref_ids, _ = one.greedy(prompts[b], steps + 1)
            assert [int(t) for t in ids[:, b]] == ref_ids[1:], b
            np.testing.assert_allclose(logits[b], _np(one.logits), rtol=0, atol=TOL)
            np.testing.assert_allclose(_np(eng.wkv[:, b]), _np(one.wkv), rtol=0, atol=TOL)
    finally:
        eng.close()
        one.close()


def test_batch_state_roundtrip_reset_and_errors():
    shape, pack = _pack("tiny", 11)
    prompts = _prompts(4, 5, shape.vocab, 11)
    eng = B200BatchEngine(pack, 4)
    try:
        _prefill(eng, prompts)
        snaps = [eng.get_state(b) for b in range(4)]
        tok = eng.logits.argmax(dim=1).tolist()
        a = eng.decode_greedy(5)
        for b in range(4):
            eng.set_state(b, snaps[b])
        eng.forward(tok)  # consume the same first ids again: step 0 of `a` used them
        b2 = eng.decode_greedy(4)
        assert np.array_equal(a[1:], b2)
        eng.reset()
        assert float(eng.wkv.abs().sum()) == 0.0
        with pytest.raises(RwkvbError):
            eng.forward([shape.vocab] * 4)
        with pytest.raises(ValueError):
            eng.forward([0] * 3)
    finally:
        eng.close()


@pytest.mark.parametrize("nb,length", [(4, 37), (5, 24), (8, 16), (40, 7)])
def test_prefill_matches_step_by_step(nb, length):
    """Chunked prefill (positions of a chunk in one GEMM) against one forward step
    per position: logits, state and the following greedy ids."""
    shape, pack = _pack("tiny", 13)
    prompts = _prompts(nb, length, shape.vocab, 13)
    a = B200BatchEngine(pack, nb)
    b = B200BatchEngine(pack, nb)
    try:
        a.prefill(prompts)
        _prefill(b, prompts)
        np.testing.assert_allclose(_np(a.logits), _np(b.logits), rtol=0, atol=TOL)
        for t_a, t_b in ((a.att_x, b.att_x), (a.wkv, b.wkv), (a.ffn_x, b.ffn_x)):
            np.testing.assert_allclose(_np(t_a), _np(t_b), rtol=0, atol=TOL)
        assert np.array_equal(a.decode_greedy(5), b.decode_greedy(5))
    finally:
        a.close()
        b.close()


def test_prefill_matches_oracle_at_0p1b_width():
    shape = synth.PRESETS["0.1b"]
    sd = synth.generate_state_dict(shape, 17, "cpu")
    pack = synth.make_pack(sd, policy="sg8")
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    nb, length = 2, 40
    prompts = _prompts(nb, length, shape.vocab, 17)
    eng = B200BatchEngine(pack, nb)
    try:
        eng.prefill(prompts)
        logits = _np(eng.logits)
        ids = eng.decode_greedy(2)
        for s in range(nb):
            ref_ids, ref_logits, _ = oracle.greedy(prompts[s], 3)
            np.testing.assert_allclose(logits[s], ref_logits[length - 1], rtol=0, atol=TOL)
            assert [int(t) for t in ids[:, s]] == ref_ids[1:]
    finally:
        eng.close()


def test_7p2b_width_engines_match_oracle():
    """7.2B width (d_model 4096, FFN 16384, 64 heads, ranks 128/128/96/480), 4 layers:
    the batch-1 persistent engine against the oracle, then chunked prefill of 8
    sessions against the batch-1 engine."""
    shape = synth.PRESETS["7.2b-l4"]
    sd = synth.generate_state_dict(shape, 23, "cuda")  # encoded on the GPU, host bytes for the oracle
    pack = synth.make_pack(sd, policy="sg8")
    del sd
    torch.cuda.empty_cache()
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    prompt = synth.seeded_prompt(3, shape.vocab, 23)
    ids_ref, logits_ref, _ = oracle.greedy(prompt, 2)
    one = B200Engine(pack)
    try:
        ids, logits = one.greedy(prompt, 2, keep_logits=True)
        assert ids == ids_ref
        np.testing.assert_allclose(_np(logits), logits_ref, rtol=0, atol=TOL)
        nb = 8
        prompts = _prompts(nb, 20, shape.vocab, 23)
        eng = B200BatchEngine(one._model, nb)
        try:
            eng.prefill(prompts)
            got = _np(eng.logits)
            for b in (0, nb - 1):
                one.reset()
                one.forward(prompts[b])
                np.testing.assert_allclose(got[b], _np(one.logits), rtol=0, atol=TOL)
        finally:
            eng.close()
    finally:
        one.close()


# ------------------------------------------------------------ LUT2 (TR2\x04) packs
def _lut2_pack(preset: str, seed: int):
    shape = synth.PRESETS[preset]
    return shape, synth.make_pack(synth.generate_state_dict(shape, seed, "cpu"), policy="lut2")


def test_lut2_batch_sessions_match_oracle():
    """Projections and head in TR2\\x04 (CUDA-core batched products): every
    session against the oracle's per-session loop."""
    shape, pack = _lut2_pack("tiny", 13)
    nb, n_new = 6, 8
    prompts = _prompts(nb, 5, shape.vocab, 13)
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    eng = B200BatchEngine(pack, nb)
    try:
        eng.prefill(prompts)  # LUT2 engines run each position as a decode step
        ids = eng.decode_greedy(n_new)
        logits = _np(eng.logits)
        for b in range(nb):
            ids_ref, logits_ref, state_ref = oracle.greedy(prompts[b], n_new + 1)
            assert [int(t) for t in ids[:, b]] == ids_ref[1:], b
            np.testing.assert_allclose(logits[b], logits_ref[-1], rtol=0, atol=TOL)
            for j, s in enumerate(eng.get_state(b)):
                np.testing.assert_allclose(_np(s).reshape(-1), state_ref[j].reshape(-1), rtol=0, atol=TOL)
    finally:
        eng.close()


@pytest.mark.parametrize("preset,nb,steps", [("0.1b", 64, 3), ("2.9b-l4", 64, 2)])
def test_lut2_batch_matches_batch1_engine(preset, nb, steps):
    shape = synth.PRESETS[preset]
    pack = synth.make_pack_streaming(shape, 6, "cuda", policy="lut2")
    prompts = _prompts(nb, 3, shape.vocab, 6)
    eng = B200BatchEngine(pack, nb)
    one = B200Engine(pack)
    try:
        _prefill(eng, prompts)
        ids = eng.decode_greedy(steps)
        logits = _np(eng.logits)
        for b in (0, 33, nb - 1):
            one.reset()
            ref_ids, _ = one.greedy(prompts[b], steps + 1)
            assert [int(t) for t in ids[:, b]] == ref_ids[1:], b
            np.testing.assert_allclose(logits[b], _np(one.logits), rtol=0, atol=TOL)
            np.testing.assert_allclose(_np(eng.wkv[:, b]), _np(one.wkv), rtol=0, atol=TOL)
    finally:
        eng.close()
        one.close()


def test_lut2_and_sg8_projections_do_not_mix():
    _, l2 = _lut2_pack("tiny", 3)
    _, sg = _pack("tiny", 3)
    mixed = dict(l2)
    mixed["head.weight"] = sg["head.weight"]
    with pytest.raises(RwkvbError):
        B200BatchEngine(mixed, 2)
    mixed = dict(sg)
    mixed["blocks.1.ffn.key.weight"] = l2["blocks.1.ffn.key.weight"]
    with pytest.raises(RwkvbError):
        B200BatchEngine(mixed, 2)


@pytest.mark.parametrize("preset,nb", [("tiny", 7), ("0.1b", 64)])
def test_lut2_tensor_core_and_cuda_core_products_agree(preset, nb):
    """The fp16 tcgen05 LUT2 GEMM (activations as two fp16 planes) against the
    fp32 CUDA-core product on the same pack and prompts: ids identical, logits
    within 1e-3."""
    shape = synth.PRESETS[preset]
    pack = synth.make_pack_streaming(shape, 8, "cuda", policy="lut2")
    prompts = _prompts(nb, 4, shape.vocab, 8)
    out = []
    for tc in (True, False):
        eng = B200BatchEngine(pack, nb, lut2_tensor_cores=tc)
        try:
            _prefill(eng, prompts)
            ids = eng.decode_greedy(4)
            out.append((ids, _np(eng.logits), _np(eng.wkv)))
        finally:
            eng.close()
    assert np.array_equal(out[0][0], out[1][0])
    np.testing.assert_allclose(out[0][1], out[1][1], rtol=0, atol=TOL)
    np.testing.assert_allclose(out[0][2], out[1][2], rtol=0, atol=TOL)
