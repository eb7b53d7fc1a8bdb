"""The ``cuda_b200`` backend end to end on the GPU, against the oracle."""

from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle.forward import OracleRWKV7  # noqa: E402
from rwkv_b200 import backend as bk  # noqa: E402
from rwkv_b200 import synth  # noqa: E402


class _ByteTokenizer:
    """Deterministic stand-in tokenizer: one id per byte."""

    def encode(self, text: str) -> list[int]:
        return list(text.encode())

    def decode(self, ids):
        return bytes(i % 256 for i in ids).decode(errors="replace")


@pytest.fixture(scope="module")
def model():
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 21, "cpu"), policy="sg8")
    oracle = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    b = bk.create_backend("cuda_b200")
    b.tokenizer = _ByteTokenizer()
    b.load_pack(None, "cuda:0")
    prov = bk.PackProvider(pack)
    b.prepare_provider(prov)
    yield shape, pack, oracle, b, prov
    b.close()


def test_generate_matches_oracle(model):
    shape, pack, oracle, b, prov = model
    text = "RWKV on B200"
    ids = b.generate(text, prov, 12, metrics=None)
    ref_ids, _, _ = oracle.greedy(list(text.encode()), 12)
    assert ids == ref_ids


def test_followup_generation_continues_the_state(model):
    shape, pack, oracle, b, prov = model
    text = "abc"
    first = b.generate(text, prov, 5, metrics=None)
    st = b.get_recurrent_state()
    more = b.decode_greedy(st, prov, 4, metrics=None)
    ref, _, _ = oracle.greedy(list(text.encode()), 9)
    assert first + more == ref


def test_callback_cancel_and_probe(model):
    shape, pack, oracle, b, prov = model
    seen = []
    st = b.prefill_text("xyz", prov, metrics=None)
    ids = b.decode_greedy(st, prov, 6, metrics=None, token_callback=seen.append)
    assert seen == ids
    logits = b.probe_logits(st)
    ref_state = oracle.zero_state()
    ref_logits = None
    for t in b"xyz":
        ref_logits = oracle.forward_token(t, ref_state)
    np.testing.assert_allclose(logits.cpu().numpy(), ref_logits, atol=1e-3, rtol=0)
    ev = threading.Event()
    ev.set()
    with pytest.raises(bk.GenerationCancelled):
        b.decode_greedy(st, prov, 3, metrics=None, cancel_event=ev)


def test_state_roundtrip_through_recurrent_state(model):
    shape, pack, oracle, b, prov = model
    st = b.prefill_text("state", prov, metrics=None)
    a = b.decode_greedy(st, prov, 5, metrics=None)
    b.set_recurrent_state(st)
    c = b.decode_greedy(st, prov, 5, metrics=None)
    assert a == c
    assert len(st.rwkv7_state) == 3 * shape.n_layer
    assert tuple(st.rwkv7_state[1].shape) == (shape.n_head, shape.head_size, shape.head_size)


def test_generate_greedy_batch_uses_batched_engine_and_matches_generate(model):
    shape, pack, oracle, b, prov = model
    prompts = ["alpha-1", "bravo-2", "charli3"]
    out = b.generate_greedy_batch(prompts, prov, 7, metrics=None)
    assert 3 in b._batch_engines  # equal-length prompts ran through the batched engine
    for p, ids in zip(prompts, out):
        ref, _, _ = oracle.greedy(list(p.encode()), 7)
        assert ids == ref
    # unequal lengths fall back to prompt-by-prompt generation with the same results
    mixed = b.generate_greedy_batch(["ab", "abcd"], prov, 4, metrics=None)
    assert mixed == [oracle.greedy(list(p.encode()), 4)[0] for p in ("ab", "abcd")]


def test_streamed_decode_is_one_launch_and_cancels_at_a_token_boundary(model):
    """With a callback the whole generation is one persistent launch whose ids
    arrive through mapped host memory; a cancel set from the callback stops it
    at the next token boundary with ``GenerationCancelled``."""
    shape, pack, oracle, b, prov = model
    assert b._engine.persistent_active
    text = "stream"
    ref, _, _ = oracle.greedy(list(text.encode()), 10)
    st = b.prefill_text(text, prov, metrics=None)
    seen = []
    ids = b.decode_greedy(st, prov, 10, metrics=None, token_callback=seen.append)
    assert ids == ref and seen == ref
    ev = threading.Event()
    got = []

    def cb(tok):
        got.append(tok)
        if len(got) == 3:
            ev.set()

    with pytest.raises(bk.GenerationCancelled):
        b.decode_greedy(st, prov, 10, metrics=None, token_callback=cb, cancel_event=ev)
    assert got == ref[:3]
    import time as _time

    with pytest.raises(bk.GenerationCancelled):
        b.decode_greedy(st, prov, 5, metrics=None, token_callback=lambda t: None, deadline=_time.monotonic() - 1)
    # the engine is usable afterwards and a fresh decode from the same state is unchanged
    assert b.decode_greedy(st, prov, 10, metrics=None) == ref


def test_long_prompt_prefill_runs_in_chunks_and_matches_oracle(model):
    shape, pack, oracle, b, prov = model
    prompt = synth.seeded_prompt(2 * b.PREFILL_CHUNK + 5, shape.vocab, 77)
    st = b.prefill_tokens(prompt)
    assert getattr(b, "_prefill_eng", None) is not None  # whole chunks went through the batched engine
    ref_ids, ref_logits, ref_state = oracle.greedy(prompt, 6)
    np.testing.assert_allclose(b.probe_logits(st).cpu().numpy(), ref_logits[len(prompt) - 1], atol=1e-3, rtol=0)
    assert b.decode_greedy(st, prov, 6, metrics=None) == ref_ids


def test_prefix_state_reuse_matches_full_prefill(model):
    """The engine's prefix cache flow: a cached prefix state continued with a
    suffix (``initial_state``) equals prefilling the whole text."""
    shape, pack, oracle, b, prov = model
    pre, suf = "system: be brief. ", "user: hi"
    st_pre = b.prefill_text(pre, prov, metrics=None)
    cached = st_pre.clone()
    st_a = b.prefill_text(suf, prov, metrics=None, initial_state=cached)
    a = b.decode_greedy(st_a, prov, 6, metrics=None)
    st_b = b.prefill_text(pre + suf, prov, metrics=None)
    c = b.decode_greedy(st_b, prov, 6, metrics=None)
    assert a == c == oracle.greedy(list((pre + suf).encode()), 6)[0]


def test_snapshot_file_resumes_the_generation(model, tmp_path):
    """State export to a reference-format snapshot file and back: the portable
    state (before the last token) resumes exactly where the live state does."""
    shape, pack, oracle, b, prov = model
    st = b.prefill_text("snap", prov, metrics=None)
    first = b.decode_greedy(st, prov, 5, metrics=None)
    live = b._last_state.clone()
    path = b.save_snapshot(tmp_path / "s.rws", prompt="snap")
    direct = b.decode_greedy(live, prov, 6, metrics=None)
    restored = b.load_snapshot(path)
    assert restored.external_state is None and restored.last_token_id == first[-1]
    resumed = b.decode_greedy(b.get_recurrent_state(), prov, 6, metrics=None)
    assert resumed == direct
    assert first + direct == oracle.greedy(list(b"snap"), 11)[0]


def test_live_state_resumes_without_a_copy_and_stale_states_are_restored(model):
    """A state the engine still holds resumes as is; a state taken before a
    later change of the engine is copied back in full: both continue exactly
    like the oracle."""
    shape, pack, oracle, b, prov = model
    text = "live"
    ref, _, _ = oracle.greedy(list(text.encode()), 7)
    st0 = b.prefill_text(text, prov, metrics=None)
    keep = st0.clone()
    calls = []
    orig = b._engine.set_state
    b._engine.set_state = lambda s: (calls.append(1), orig(s))[1]
    try:
        a = b.decode_greedy(st0, prov, 3, metrics=None)  # the engine holds st0: no copy
        assert calls == []
        st1 = b._last_state
        c = b.decode_greedy(st1, prov, 4, metrics=None)  # live again
        assert calls == []
        assert a + c == ref
        again = b.decode_greedy(keep, prov, 7, metrics=None)  # stale: restored in full
        assert calls == [1]
        assert again == ref
    finally:
        b._engine.set_state = orig
