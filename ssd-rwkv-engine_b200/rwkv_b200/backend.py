"""``cuda_b200``: the drop-in pack backend of the reference engine's plugin API.

Mirrors, method for method, the reference's ``PackBackend`` contract
(``rwkv_ssd/backends/pack_backend.py:18-165``, ``base.py:11-67``) as the
Albatross adapter implements it (``rwkv_ssd/backends/albatross.py:715-1015``):

* ``load_pack(manifest, device)``   — remember the pack layout and target GPU
* ``prepare_provider(provider, *, config)`` — copy every packed blob once from
  the provider into HBM and build the fused decode engine
* ``prefill_text`` / ``prefill_tokens`` -> ``RecurrentState``
* ``decode_greedy(state, provider, max_tokens, metrics, *, temperature,
  token_callback, cancel_event, deadline)`` -> token ids
* ``generate`` / ``generate_greedy`` / ``generate_greedy_batch``
* ``get_recurrent_state`` / ``set_recurrent_state`` / ``probe_logits``
* ``capabilities()``

``RecurrentState`` keeps the reference layout (``state_cache.py:38-56``):
``rwkv7_state`` is the 3-tensors-per-layer list ``[x_prev_att, S, x_prev_ffn]``
(device tensors here); the pending next-token logits ride in
``external_state`` like the Albatross backend's ``pending_logits``.

Providers: any object exposing the reference ``ManifestWeightProvider``'s
``manifest`` + ``_read_packed_bytes(entry, timing)`` (raw pack bytes per
``TensorEntry``), or this module's in-memory ``PackProvider``.
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from .synth import PackedTensor

CUDA_B200_BACKENDS = frozenset({"cuda_b200", "b200"})
SUPPORTED_CODECS = ("none", "scale_u8_grouped", "trinity_lut2")


try:
    # Inside the reference tree the backend uses the reference's own types, so
    # its engine's isinstance checks (``is_pack_backend``), ``except`` clauses
    # and state cache see this backend's objects as their own.
    from rwkv_ssd.backends.pack_backend import PackBackend as _PackBase
    from rwkv_ssd.runtime.errors import BackendNotAvailableError, CapabilityNotSupportedError
    from rwkv_ssd.runtime.generation_control import GenerationCancelled
    from rwkv_ssd.runtime.state_cache import RecurrentState

    REFERENCE_TYPES = True
except ImportError:
    REFERENCE_TYPES = False
    _PackBase = object

    class BackendNotAvailableError(Exception):
        """Mirror of ``rwkv_ssd.runtime.errors.BackendNotAvailableError``."""

    class CapabilityNotSupportedError(Exception):
        """Mirror of ``rwkv_ssd.runtime.errors.CapabilityNotSupportedError``."""

        def __init__(self, capability: str, backend: str, detail: str | None = None):
            self.capability = str(capability)
            self.backend = str(backend)
            msg = f"backend {self.backend!r} does not support capability {self.capability!r}"
            super().__init__(msg + (f": {detail}" if detail else ""))

    class GenerationCancelled(RuntimeError):
        """Mirror of ``rwkv_ssd.runtime.generation_control.GenerationCancelled``."""

    @dataclass
    class RecurrentState:
        """Field-compatible with the reference ``RecurrentState`` (state_cache.py:38-56)."""

        last_token_id: int = 0
        h: torch.Tensor | None = None
        rwkv7_state: list[torch.Tensor] | None = None
        external_state: object | None = None

        def clone(self) -> "RecurrentState":
            ext = self.external_state
            if isinstance(ext, dict):
                ext = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in ext.items()}
            return RecurrentState(int(self.last_token_id), self.h.clone() if self.h is not None else None,
                                  [t.clone() for t in self.rwkv7_state] if self.rwkv7_state is not None else None,
                                  ext)


class _Control:
    """Token-boundary cancellation / deadline / callback (generation_control.py:19-35)."""

    def __init__(self, token_callback=None, cancel_event=None, deadline=None):
        self.cb, self.cancel, self.deadline = token_callback, cancel_event, deadline

    def check(self) -> None:
        if self.cancel is not None and self.cancel.is_set():
            raise GenerationCancelled("generation cancelled")
        if self.deadline is not None and time.monotonic() >= self.deadline:
            raise GenerationCancelled("generation deadline exceeded")

    def emit(self, tok: int) -> None:
        self.check()
        if self.cb is not None:
            self.cb(int(tok))


def _control(token_callback=None, cancel_event=None, deadline=None):
    if token_callback is None and cancel_event is None and deadline is None:
        return None
    return _Control(token_callback, cancel_event, deadline)


# ---------------------------------------------------------------- providers
_DEQUANT_CODEC = {"scale_u8_grouped": "sg8", "trinity_lut2": "lut2", "none": "none"}
_DTYPES = {"float32": np.float32, "float16": np.float16, "bfloat16": "bf16"}


@dataclass
class _Entry:
    name: str
    shape: list
    dtype: str = "float32"
    dequant: str = "none"
    layer_id: int = -1


class PackProvider:
    """In-memory pack provider (name -> ``PackedTensor``) with the reference
    provider's fused-blob protocol (``weight_provider.py:660-667``)."""

    def __init__(self, pack: dict[str, PackedTensor]):
        self.pack = pack
        self._fused = {n: (e.payload, int(e.shape[0]), int(e.shape[1])) for n, e in pack.items()
                       if e.codec in ("sg8", "lut2")}

    def packed_tensors(self) -> dict[str, PackedTensor]:
        return self.pack

    def _use_fused_lut_matmul(self) -> bool:
        return True

    def get_fused_lut_blob(self, name: str):
        return self._fused.get(name)


def packed_tensors_from_provider(provider) -> dict[str, PackedTensor]:
    """Raw packed tensors from a provider (in-memory or the reference's)."""
    if hasattr(provider, "packed_tensors"):
        return provider.packed_tensors()
    manifest = getattr(provider, "manifest", None) or getattr(provider, "_manifest", None)
    reader = getattr(provider, "_read_packed_bytes", None)
    if manifest is None or not callable(reader):
        raise TypeError("provider exposes neither packed_tensors() nor manifest + _read_packed_bytes()")
    out: dict[str, PackedTensor] = {}
    for entry in manifest.tensors:
        raw = reader(entry, None)
        dq = (entry.dequant or "none").strip().lower()
        if dq not in _DEQUANT_CODEC:
            raise CapabilityNotSupportedError("codec", "CudaB200Backend", f"{entry.name}: {dq}")
        codec = _DEQUANT_CODEC[dq]
        shape = tuple(int(d) for d in entry.shape)
        if codec == "none":
            dt = _DTYPES.get(str(entry.dtype), np.float32)
            if dt == "bf16":
                u16 = np.frombuffer(bytes(raw), dtype=np.uint16).astype(np.uint32) << 16
                vals = u16.view(np.float32)
            else:
                vals = np.frombuffer(bytes(raw), dtype=dt).astype(np.float32)
            out[entry.name] = PackedTensor(entry.name, shape, "none", vals.reshape(-1).copy())
        else:
            if codec == "lut2" and bytes(raw[:3]) != b"TR2":
                raise CapabilityNotSupportedError("codec", "CudaB200Backend", f"{entry.name}: per-tensor LUT2")
            if len(shape) != 2:
                shape = (1, int(np.prod(shape)))
            out[entry.name] = PackedTensor(entry.name, shape, codec, bytes(raw))
    return out


# ----------------------------------------------------------------- backend
class CudaB200Backend(_PackBase):
    """RWKV-7 packed decode on one B200 through the sm_100a library.

    Subclasses the reference's ``PackBackend`` when the reference package is
    importable (its engine then routes it through ``_generate_pack``), else
    stands alone with the same method set."""

    supports_streaming: bool = True

    def __init__(self, tokenizer: Any | None = None, *, use_graph: bool = True):
        self.tokenizer = tokenizer
        self.use_graph = use_graph
        self._manifest = None
        self._device = torch.device("cuda", 0)
        self._engine = None
        self._model = None
        self._batch_engines: dict[int, Any] = {}
        self._last_state: RecurrentState | None = None
        self._lock = threading.Lock()
        self._epoch = 0  # moved by every change of the engine's state (see _snapshot)

    # -------------------------------------------------------- RecurrentBackend
    def load(self, model_path: str, strategy: str, device: str) -> None:
        self.capability_error("checkpoint_load", "cuda_b200 consumes runtime packs via load_pack()")

    def load_pack(self, manifest, device: str) -> None:
        self._manifest = manifest
        dev = torch.device(device if device not in ("auto", "", None) else "cuda")
        if dev.type != "cuda":
            raise BackendNotAvailableError(f"cuda_b200 needs a CUDA device, got {device!r}")
        self._device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())

    def prepare_provider(self, provider, *, config: Any = None) -> None:
        from .engine import B200Engine

        if self._engine is not None:
            return
        if not torch.cuda.is_available():
            raise BackendNotAvailableError("cuda_b200 needs a CUDA device")
        from .engine import ModelUpload

        pack = packed_tensors_from_provider(provider)
        budget, resident, slots = self._residency(config, pack)
        with torch.cuda.device(self._device):
            self._model = ModelUpload(pack, self._device, hbm_budget=budget, resident_layers=resident,
                                      stage_slots=slots)
        self._engine = B200Engine(self._model, device=self._device, use_graph=self.use_graph)
        self._epoch += 1

    @staticmethod
    def _residency(config, pack) -> tuple[int | None, list[int] | None, int]:
        """Residency tiers from the engine config (``RuntimeConfig.mode`` and
        ``residency_profile``, as the reference's ``apply_residency_policy``,
        residency.py:13-44): "resident" keeps every layer in HBM, "partial" the
        profile's ``resident_layer_ids`` (default: the first and last layers),
        "streaming" none; an ``hbm_budget_bytes`` attribute keeps as many layers
        as fit in that many bytes of HBM.  ``stage_slots`` (default 2) device
        slots receive the streamed layers."""
        if config is None:
            return None, None, 2
        slots = int(getattr(config, "stage_slots", 2) or 2)
        budget = getattr(config, "hbm_budget_bytes", None)
        if budget is not None:
            return int(budget), None, slots
        mode = str(getattr(config, "mode", "resident") or "resident").strip().lower()
        n_layer = 1 + max(int(n.split(".")[1]) for n in pack if n.startswith("blocks."))
        if mode == "streaming":
            return None, [], slots
        if mode == "partial":
            prof = getattr(config, "residency_profile", None)
            if prof:
                import json
                from pathlib import Path

                ids = json.loads(Path(prof).read_text(encoding="utf-8")).get("resident_layer_ids", [])
                return None, [int(i) for i in ids], slots
            return None, sorted({0, n_layer - 1}), slots
        return None, None, slots

    @property
    def num_layers(self) -> int:
        if self._engine is not None:
            return self._engine.shape.n_layer
        if self._manifest is not None:
            return 1 + max(int(e.name.split(".")[1]) for e in self._manifest.tensors if e.name.startswith("blocks."))
        return 0

    def decode_text(self, token_ids: list[int]) -> str:
        if self.tokenizer is not None and hasattr(self.tokenizer, "decode"):
            return self.tokenizer.decode(list(token_ids))
        return " ".join(str(int(t)) for t in token_ids)

    def capability_error(self, capability: str, detail: str | None = None) -> None:
        raise CapabilityNotSupportedError(capability, type(self).__name__, detail)

    def capabilities(self) -> dict[str, object]:
        return {
            "name": "cuda_b200",
            "declared": {
                "pack_streaming": True, "skeleton": False, "resident": True, "state_snapshot": True,
                "batch": True, "prefix_cache": False, "tokenizer": self.tokenizer is not None,
                "state_kind": "rwkv7", "supported_codecs": list(SUPPORTED_CODECS), "requires_ggml_bin": False,
                "token_generation": True, "logits_probe": True, "state_transfer": True,
                "followup_generation": True, "sampling": True, "incremental_streaming": True,
                "cancellation": True, "deadlines": True, "process_workers": False,
                "native_layer_streaming": False, "native_cached_layer_step": True,
                "deepembed": False, "deepembed_streaming": False,
            },
            "runtime": {"loaded": self._engine is not None, "device": str(self._device)},
        }

    def supports_capability(self, capability: str) -> bool:
        return bool(self.capabilities()["declared"].get(capability, False))

    # ---------------------------------------------------------------- state
    def _engine_or_raise(self):
        if self._engine is None:
            raise RuntimeError("cuda_b200: call prepare_provider() before generating")
        return self._engine

    # Two forms of RecurrentState.  The *live* form (what prefill and decode
    # return) holds the state after every consumed token in rwkv7_state and,
    # in external_state, the next token's logits ("pending_logits") plus the
    # state before the last token ("pre_state").  The *portable* form (what
    # get_recurrent_state returns and snapshot files hold) is the reference's:
    # rwkv7_state = the state before last_token_id, nothing else; resuming
    # consumes last_token_id first (rwkv7_forward.py:941-990).
    #
    # A live state also carries ("engine_epoch") the backend and the epoch at
    # which it was taken.  Every operation that changes the engine's state
    # moves the epoch first, so a state whose mark equals the current epoch is
    # exactly what the engine holds and resuming it copies nothing.
    def _snapshot(self, last: int, pre: list[torch.Tensor]) -> RecurrentState:
        eng = self._engine
        self._epoch += 1
        return RecurrentState(last_token_id=int(last), rwkv7_state=eng.get_state(),
                              external_state={"pending_logits": eng.logits.clone(), "pre_state": pre,
                                              "engine_epoch": (id(self), self._epoch)})

    def _restore(self, state: RecurrentState) -> list[torch.Tensor]:
        """Load ``state`` into the engine (consuming ``last_token_id`` for the
        portable form); returns the state before the last token."""
        eng = self._engine
        if state.rwkv7_state is None:
            raise ValueError("cuda_b200 state has no rwkv7_state")
        ext = state.external_state if isinstance(state.external_state, dict) else {}
        pl = ext.get("pending_logits")
        if pl is not None and ext.get("engine_epoch") == (id(self), self._epoch):
            pre = ext.get("pre_state")
            return list(pre) if pre is not None else eng.get_state()
        self._epoch += 1
        if pl is not None:
            eng.set_state(state.rwkv7_state)
            eng.logits.copy_(pl.to(eng.device, torch.float32))
            pre = ext.get("pre_state")
            return [t.clone() for t in pre] if pre is not None else eng.get_state()
        eng.set_state(state.rwkv7_state)
        pre = eng.get_state()
        eng.forward([int(state.last_token_id)])
        return pre

    def get_recurrent_state(self) -> RecurrentState | None:
        """The portable form of the current state (single representation, as
        the reference's snapshot writer requires)."""
        st = self._last_state
        if st is None:
            return None
        ext = st.external_state if isinstance(st.external_state, dict) else {}
        pre = ext.get("pre_state")
        if pre is None:
            return st.clone()
        return RecurrentState(last_token_id=int(st.last_token_id), rwkv7_state=[t.clone() for t in pre])

    def save_snapshot(self, path, *, prompt: str = "", state: RecurrentState | None = None):
        """Write the current (or the given) state as a reference-format snapshot
        file (``rwkv_b200.snapshot``); the reference engine's load_snapshot
        reads it, and load_snapshot here reads the reference's."""
        from . import snapshot

        st = state if state is not None else self.get_recurrent_state()
        if st is None:
            raise RuntimeError("cuda_b200 has no recurrent state to snapshot")
        ext = st.external_state if isinstance(st.external_state, dict) else {}
        pre = ext.get("pre_state") if ext.get("pending_logits") is not None else None
        tensors = pre if pre is not None else st.rwkv7_state
        meta = snapshot.SnapshotMeta(prompt=prompt, last_token_id=int(st.last_token_id))
        return snapshot.save_snapshot(path, tensors, meta)

    def load_snapshot(self, path) -> RecurrentState:
        """Read a snapshot file (this backend's or the reference engine's) and
        make it the current state (portable form)."""
        from . import snapshot

        tensors, meta = snapshot.load_snapshot(path)
        st = RecurrentState(last_token_id=int(meta.last_token_id), rwkv7_state=tensors)
        self.set_recurrent_state(st)
        return st.clone()

    def set_recurrent_state(self, state: RecurrentState) -> None:
        if state.rwkv7_state is None or len(state.rwkv7_state) != 3 * self.num_layers:
            raise ValueError("cuda_b200 state has an incompatible representation")
        self._last_state = state.clone()

    def probe_logits(self, state: RecurrentState | None = None):
        cur = state or self._last_state
        if cur is None or not isinstance(cur.external_state, dict):
            return None
        pl = cur.external_state.get("pending_logits")
        return pl.detach().clone() if pl is not None else None

    # ------------------------------------------------------------- prefill
    def _encode(self, text: str) -> list[int]:
        if self.tokenizer is None:
            raise CapabilityNotSupportedError("tokenizer", "CudaB200Backend",
                                              "construct with a tokenizer or call prefill_tokens()")
        enc = self.tokenizer.encode(text)
        return list(getattr(enc, "ids", enc))

    def prefill_tokens(self, token_ids: list[int], initial_state: RecurrentState | None = None, *,
                       metrics: Any = None, cancel_event=None, deadline=None) -> RecurrentState:
        eng = self._engine_or_raise()
        ctl = _control(cancel_event=cancel_event, deadline=deadline)
        t0 = time.perf_counter()
        with self._lock:
            if initial_state is not None:
                self._restore(initial_state)
            self._epoch += 1
            if initial_state is None:
                eng.reset()
            ids = [int(t) for t in token_ids] or [0]
            done = self._chunked_prefill(ids[:-1], ctl)
            rest = ids[done:-1]
            if ctl is None:
                if rest:
                    eng.forward(rest)
            else:
                for t in rest:
                    ctl.check()
                    eng.forward([t])
            pre = eng.get_state()  # the state before the last prompt token (portable form)
            if ctl is not None:
                ctl.check()
            eng.forward([ids[-1]])
            state = self._snapshot(ids[-1], pre)
        torch.cuda.synchronize(eng.device)
        if metrics is not None and hasattr(metrics, "prefill_wall_s"):
            metrics.prefill_wall_s = time.perf_counter() - t0
        self._last_state = state
        return state.clone()

    PREFILL_CHUNK = 64  # positions per tcgen05 GEMM of the one-session prefill

    def _chunked_prefill(self, ids: list[int], ctl) -> int:
        """Whole ``PREFILL_CHUNK``-position chunks of a prompt through the
        batched engine at one session (every projection of a chunk is one
        tcgen05 GEMM over its positions, ``rwkvb_batch_prefill``), continuing
        from and returning to the batch-1 engine's state; returns how many
        prompt tokens it consumed (0 when the prompt is shorter than a chunk or
        a projection is not SG8).  The rest of the prompt runs on the batch-1
        engine.  Mirrors the reference's chunked prompt prefill
        (rwkv7_forward.py:1046-1175)."""
        P = self.PREFILL_CHUNK
        full = len(ids) // P * P
        if full == 0 or not self._model.sg8_projections:
            return 0
        from .engine import B200BatchEngine

        eng = self._engine
        pe = getattr(self, "_prefill_eng", None)
        if pe is None:
            pe = B200BatchEngine(self._model, 1, device=self._device)
            self._prefill_eng = pe
        pe.set_state(0, eng.get_state())
        if ctl is None:
            pe.prefill([ids[:full]])
        else:
            for c0 in range(0, full, P):
                ctl.check()
                pe.prefill([ids[c0:c0 + P]])
        eng.att_x.copy_(pe.att_x[:, 0])
        eng.wkv.copy_(pe.wkv[:, 0])
        eng.ffn_x.copy_(pe.ffn_x[:, 0])
        eng.logits.copy_(pe.logits[0])
        return full

    def prefill_text(self, text: str, provider, metrics, initial_state: RecurrentState | None = None, *,
                     cancel_event=None, deadline=None) -> RecurrentState:
        self.prepare_provider(provider)
        return self.prefill_tokens(self._encode(text), initial_state, metrics=metrics, cancel_event=cancel_event,
                                   deadline=deadline)

    # -------------------------------------------------------------- decode
    def decode_greedy(self, state: RecurrentState, provider, max_tokens: int, metrics, *, temperature: float = 0.0,
                      token_callback=None, cancel_event=None, deadline=None) -> list[int]:
        """Greedy (or sampled, ``temperature > 0``) continuation of ``state``.

        Greedy decoding is ONE device launch for the whole generation: without
        a callback/cancel/deadline the ids come back at the end; with them the
        persistent kernel streams each id into mapped pinned host memory as it
        is made, the callback runs on this thread as ids arrive, and a set
        ``cancel_event`` or a passed ``deadline`` sets the device's cancel word
        (the decode stops at the next token boundary and ``GenerationCancelled``
        is raised, as the reference's token-boundary checks do).  The state
        ends after every emitted token, with the next token's logits pending."""
        self.prepare_provider(provider)
        eng = self._engine_or_raise()
        n = max(0, int(max_tokens))
        ctl = _control(token_callback, cancel_event, deadline)
        out: list[int] = []
        with self._lock:
            pre = self._restore(state)
            self._epoch += 1
            t0 = time.perf_counter()
            if n and float(temperature) <= 0.0 and (ctl is None or eng.persistent_active):
                first = int(torch.argmax(eng.logits).item())
                if ctl is None:
                    # step i consumes emitted token i: n - 1 steps on the
                    # device, the state before the last emitted token is kept
                    # (portable form), then the last token is consumed
                    out = [first] + (eng.decode_greedy(first, n - 1) if n > 1 else [])
                    pre = eng.get_state()
                    eng.forward([out[-1]])
                    lat = (time.perf_counter() - t0) * 1e3 / n
                    self._record(metrics, [lat] * n)
                else:
                    lats: list[float] = []
                    last = [time.perf_counter()]

                    def emit(tok: int) -> None:
                        ctl.emit(tok)
                        out.append(int(tok))
                        now = time.perf_counter()
                        lats.append((now - last[0]) * 1e3)
                        last[0] = now

                    emit(first)

                    def on_token(i: int, tok: int) -> None:
                        emit(tok)

                    def should_stop() -> bool:
                        try:
                            ctl.check()
                        except GenerationCancelled:
                            return True
                        return False

                    if n > 1:
                        eng.decode_stream(first, n - 1, on_token=on_token, should_stop=should_stop)
                    if len(out) < n:  # stopped at a token boundary by the cancel word
                        self._record(metrics, lats)
                        ctl.check()
                        raise GenerationCancelled("generation cancelled")
                    pre = eng.get_state()
                    eng.forward([out[-1]])
                    self._record(metrics, lats)
            else:
                lats = []
                for _ in range(n):
                    if ctl is not None:
                        ctl.check()
                    s0 = time.perf_counter()
                    tok = self._sample(eng.logits, float(temperature))
                    out.append(tok)
                    pre = eng.get_state()
                    eng.forward([tok])
                    if ctl is not None:
                        ctl.emit(tok)
                    lats.append((time.perf_counter() - s0) * 1e3)
                self._record(metrics, lats)
            self._last_state = self._snapshot(out[-1] if out else state.last_token_id, pre)
        return out

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float) -> int:
        if temperature <= 0.0:
            return int(torch.argmax(logits).item())
        probs = torch.softmax(logits.float() / temperature, dim=-1)
        probs = torch.nan_to_num(probs, nan=0.0, posinf=0.0, neginf=0.0)
        if not bool(torch.isfinite(probs.sum())) or float(probs.sum()) <= 0.0:
            return int(torch.argmax(logits).item())
        return int(torch.multinomial(probs, 1).item())

    @staticmethod
    def _record(metrics, lats: list[float]) -> None:
        if metrics is None:
            return
        tl = getattr(metrics, "token_latencies_ms", None)
        if isinstance(tl, list):
            tl.extend(lats)
        if hasattr(metrics, "tokens_generated"):
            metrics.tokens_generated = len(lats)
        if hasattr(metrics, "ttft_s") and lats and getattr(metrics, "ttft_s", 0.0) <= 0.0:
            metrics.ttft_s = lats[0] / 1e3

    # ---------------------------------------------------------- generation
    def generate(self, prompt: str, provider, max_tokens: int, metrics, *, temperature: float = 0.0,
                 greedy: bool = True, token_callback=None, cancel_event=None, deadline=None) -> list[int]:
        ctl = _control(token_callback, cancel_event, deadline)
        if ctl is not None:
            ctl.check()
        state = self.prefill_text(prompt, provider, metrics, cancel_event=cancel_event, deadline=deadline)
        if ctl is not None:
            ctl.check()
        return self.decode_greedy(state, provider, max_tokens, metrics, temperature=0.0 if greedy else temperature,
                                  token_callback=token_callback, cancel_event=cancel_event, deadline=deadline)

    def generate_tokens(self, prompt: str, provider, max_tokens: int, metrics, *, temperature: float = 0.0,
                        greedy: bool = True, token_callback=None, cancel_event=None, deadline=None) -> list[int]:
        return self.generate(prompt, provider, max_tokens, metrics, temperature=temperature, greedy=greedy,
                             token_callback=token_callback, cancel_event=cancel_event, deadline=deadline)

    def generate_greedy(self, prompt: str, provider, max_tokens: int, metrics) -> list[int]:
        return self.generate(prompt, provider, max_tokens, metrics)

    def generate_greedy_batch(self, prompts: list[str], provider, max_tokens: int, metrics) -> list[list[int]]:
        """Greedy ids for every prompt.  Prompts of equal token length (up to 64,
        SG8 projections) decode together through the batched engine (one step
        advances every session); other batches run prompt by prompt.  Each
        session's ids equal those of ``generate`` on that prompt alone."""
        self.prepare_provider(provider)
        ids = [self._encode(p) for p in prompts]
        n = max(0, int(max_tokens))
        if not ids:
            return []
        same = len({len(t) for t in ids}) == 1 and len(ids[0]) > 0
        if not (same and 2 <= len(ids) <= 64 and n > 0 and self._model.sg8_projections):
            return [self.generate(p, provider, max_tokens, metrics) for p in prompts]
        from .engine import B200BatchEngine

        nb = len(ids)
        with self._lock:
            eng = self._batch_engines.get(nb)
            if eng is None:
                eng = B200BatchEngine(self._model, nb, device=self._device)
                self._batch_engines[nb] = eng
            t0 = time.perf_counter()
            eng.reset()
            eng.prefill(ids)  # chunks of positions as tcgen05 GEMM rows (rwkvb_batch_prefill)
            first = eng.logits.argmax(dim=1).tolist()
            rest = eng.decode_greedy(n - 1) if n > 1 else np.zeros((0, nb), np.int32)
            torch.cuda.synchronize(self._device)
            if metrics is not None and hasattr(metrics, "tokens_generated"):
                metrics.tokens_generated = n * nb
            if metrics is not None and hasattr(metrics, "decode_wall_s"):
                metrics.decode_wall_s = time.perf_counter() - t0
        return [[int(first[b])] + [int(v) for v in rest[:, b]] for b in range(nb)]

    def close(self) -> None:
        for eng in self._batch_engines.values():
            eng.close()
        self._batch_engines = {}
        pe = getattr(self, "_prefill_eng", None)
        if pe is not None:
            pe.close()
            self._prefill_eng = None
        if self._engine is not None:
            self._engine.close()
            self._engine = None
            self._epoch += 1
        self._model = None


# ------------------------------------------------------------- factory
def create_backend(name: str):
    """Mirror of ``create_backend`` (``backends/factory.py:32-46``) for this backend's keys."""
    key = name.lower().strip()
    if key in CUDA_B200_BACKENDS:
        return CudaB200Backend()
    raise ValueError(f"Unknown backend {name!r}. Choose: cuda_b200 (B200 sm_100a packed decode).")


def ensure_v0_backend(name: str) -> None:
    """Availability gate like ``ensure_v0_backend`` (``backends/factory.py:60-78``)."""
    key = name.lower().strip()
    if key not in CUDA_B200_BACKENDS:
        raise ValueError(f"Unknown backend {name!r}")
    if not torch.cuda.is_available():
        raise BackendNotAvailableError(f"Backend {name!r} requires a CUDA device (B200, sm_100a).")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        raise BackendNotAvailableError(f"Backend {name!r} is built for sm_100a; device is sm_{major}{minor}.")
    from . import native

    native.lib()
