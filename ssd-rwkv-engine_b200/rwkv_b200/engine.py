"""Host wrapper of the device decode engine (``rwkvb_engine_*`` in the C ABI).

``B200Engine`` takes a packed RWKV-7 model — a mapping ``name -> entry`` with
``codec`` (``"sg8"``, ``"lut2"`` or ``"none"``), ``payload`` (wire blob as
bytes / uint8 tensor, or fp32 values) and checkpoint ``shape`` — uploads it to
HBM once (``residency.WeightArena``) and drives the fused token step.

It replaces, per token, the reference's embedding + ``ln0``
(``rwkv7_skeleton.py:74-81``), ``forward_block_packed`` for every layer
(``packed_block_forward.py:76-166``), ``ln_out`` + packed head
(``rwkv7_forward.py:791-809``) and greedy argmax (``sampling.py:161-163``).
The recurrent state keeps the reference ``RecurrentState.rwkv7_state`` layout
(``state_cache.py:38-56``): per layer ``[x_prev_att (C), S (H, N, N), x_prev_ffn (C)]``.
"""

from __future__ import annotations

import ctypes
import re
import time

import numpy as np
import torch

from . import native
from .residency import LayerStaging, VectorArena, WeightArena, _place, layer_of, plan_residency
from .synth import RWKV7Shape

_MATS = ("att.receptance.weight", "att.key.weight", "att.value.weight", "att.output.weight",
         "att.w1", "att.w2", "att.a1", "att.a2", "att.g1", "att.g2", "att.v1", "att.v2",
         "ffn.key.weight", "ffn.value.weight")
_DESC_FIELD = {"att.receptance.weight": "att_r", "att.key.weight": "att_k", "att.value.weight": "att_v",
               "att.output.weight": "att_o", "att.w1": "w1", "att.w2": "w2", "att.a1": "a1", "att.a2": "a2",
               "att.g1": "g1", "att.g2": "g2", "att.v1": "v1", "att.v2": "v2",
               "ffn.key.weight": "ffn_key", "ffn.value.weight": "ffn_value"}
_VEC_FIELD = {"ln1.weight": "ln1_w", "ln1.bias": "ln1_b", "ln2.weight": "ln2_w", "ln2.bias": "ln2_b",
              "att.x_r": "x_r", "att.x_w": "x_w", "att.x_k": "x_k", "att.x_v": "x_v", "att.x_a": "x_a",
              "att.x_g": "x_g", "att.w0": "w0", "att.a0": "a0", "att.v0": "v0", "att.k_k": "k_k",
              "att.k_a": "k_a", "att.ln_x.weight": "lnx_w", "att.ln_x.bias": "lnx_b", "ffn.x_k": "ffn_x_k"}


class _CudaArray:
    """Expose a raw device pointer to torch via ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def infer_shape(pack) -> RWKV7Shape:
    """Model dimensions from checkpoint tensor shapes."""
    L = 1 + max(int(m.group(1)) for n in pack if (m := re.match(r"blocks\.(\d+)\.", n)))
    V, C = pack["emb.weight"].shape
    H, N = pack["blocks.0.att.r_k"].shape
    F = pack["blocks.0.ffn.key.weight"].shape[0]
    rw = pack["blocks.0.att.w1"].shape[1]
    ra = pack["blocks.0.att.a1"].shape[1]
    rv = pack["blocks.1.att.v1"].shape[1] if L > 1 else pack["blocks.0.att.v1"].shape[1]
    rg = pack["blocks.0.att.g1"].shape[1]
    return RWKV7Shape(L, int(C), int(N), int(F), int(V), int(rw), int(ra), int(rv), int(rg))


class ModelUpload:
    """A packed model in HBM plus its ``rwkvb_model_desc`` (weights in one
    ``WeightArena``, fp32 vectors in one ``VectorArena``).

    Residency tiers: with ``hbm_budget`` (bytes of packed weights) below the
    model's size, or an explicit ``resident_layers`` list, the layers that do
    not fit stay in pinned host memory and ``stage`` (a ``LayerStaging``)
    streams them through ``stage_slots`` device slots on every token step; the
    embedding, the head and the kept ("hot") layers are resident."""

    def __init__(self, pack, device: torch.device, *, hbm_budget: int | None = None, stage_slots: int = 2,
                 resident_layers: list[int] | None = None):
        s = infer_shape(pack)
        self.shape = s
        self.device = device
        proj = ("att.receptance.weight", "att.key.weight", "att.value.weight", "att.output.weight",
                "ffn.key.weight", "ffn.value.weight")
        self.sg8_projections = all(e.codec == "sg8" for n, e in pack.items() if n.endswith(proj) or n == "head.weight")
        mats, vecs = [], {}
        for name, e in pack.items():
            if e.codec in ("sg8", "lut2"):
                mats.append((name, e.payload, (int(e.shape[0]), int(e.shape[1])), e.codec))
            else:
                vecs[name] = np.asarray(e.payload, dtype=np.float32).reshape(-1) \
                    if not isinstance(e.payload, torch.Tensor) else e.payload
        # per-layer matrices (r_k is decoded into a vector at load: always resident)
        by_layer: dict[int, list] = {li: [] for li in range(s.n_layer)}
        globals_ = []
        for it in mats:
            li = layer_of(it[0])
            (by_layer[li] if li >= 0 and not it[0].endswith(".att.r_k") else globals_).append(it)
        streamed = plan_residency({li: _place(v)[2] for li, v in by_layer.items()}, _place(globals_)[2], s.n_layer,
                                  hbm_budget=hbm_budget, n_slots=stage_slots, resident_layers=resident_layers)
        resident = globals_ + [it for li in range(s.n_layer) if li not in set(streamed) for it in by_layer[li]]
        self.stage = LayerStaging(by_layer, streamed, s.n_layer, stage_slots, device) if streamed else None
        self.weights = WeightArena(resident, device)
        self.vectors = VectorArena(vecs, device)
        for i in range(s.n_layer):
            nm = f"blocks.{i}.att.r_k"
            if nm in self.weights:
                self.vectors.add_decoded(nm, self.weights[nm])
        torch.cuda.synchronize(device)
        self.layers = (native.LayerDesc * s.n_layer)()
        for i in range(s.n_layer):
            d = self.layers[i]
            for suffix in _MATS:
                name = f"blocks.{i}.{suffix}"
                if name in self.weights:
                    setattr(d, _DESC_FIELD[suffix], self.weights[name].desc)
                elif self.stage is not None and name in self.stage.descs:
                    setattr(d, _DESC_FIELD[suffix], self.stage.descs[name].desc)
            for suffix, field in _VEC_FIELD.items():
                name = f"blocks.{i}.{suffix}"
                if name in self.vectors.offs or name in self.vectors.extra:
                    setattr(d, field, self.vectors.ptr(name))
            d.r_k = self.vectors.ptr(f"blocks.{i}.att.r_k")
        md = native.ModelDesc()
        md.n_layer, md.n_embd, md.head_size, md.ffn, md.vocab = s.n_layer, s.n_embd, s.head_size, s.ffn, s.vocab
        md.emb = self.weights["emb.weight"].desc
        md.head = self.weights["head.weight"].desc
        md.ln0_w = self.vectors.ptr("blocks.0.ln0.weight")
        md.ln0_b = self.vectors.ptr("blocks.0.ln0.bias")
        md.ln_out_w = self.vectors.ptr("ln_out.weight")
        md.ln_out_b = self.vectors.ptr("ln_out.bias")
        md.layers = self.layers
        self.md = md


class B200Engine:
    """A packed RWKV-7 model resident on one GPU, decoded by the fused engine.

    ``pack`` is the packed model, or a ``ModelUpload`` already resident on the
    device (shared with a ``B200BatchEngine``)."""

    def __init__(self, pack, *, device: int | torch.device = 0, use_graph: bool = True,
                 prefetch_distance: int | None = None, persistent: bool = True, trace: bool = False,
                 l2_policy: bool = True, ring_slots: int | None = None, ffn_chunk_order: bool = True,
                 extra_flags: int = 0):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("B200Engine needs a CUDA device; there is no CPU path")
        self.lib = native.lib()
        with torch.cuda.device(self.device):
            self._model = pack if isinstance(pack, ModelUpload) else ModelUpload(pack, self.device)
            self.shape = s = self._model.shape
            md = self._model.md
            flags = 0 if use_graph else native.FLAG_NO_GRAPH
            if not persistent:
                flags |= native.FLAG_NO_PERSISTENT
            if trace:
                flags |= native.FLAG_TRACE
            if not l2_policy:
                flags |= native.FLAG_NO_L2_POLICY
            if prefetch_distance is not None:
                flags |= native.FLAG_EXPLICIT_PREFETCH | ((int(prefetch_distance) & 0xF) << 4)
            if ring_slots is not None:
                flags |= (int(ring_slots) & 0xF) << native.FLAG_RING_SLOTS_SHIFT
            if not ffn_chunk_order:
                flags |= native.FLAG_FFN_ROW_ORDER
            flags |= int(extra_flags)  # further rwkvb_engine_create flag bits (include/rwkv_b200.h)
            h = ctypes.c_void_p()
            if self._model.stage is not None:
                # streamed layers: the multi-kernel step with the staging copies in it
                native.check(self.lib.rwkvb_engine_create_staged(ctypes.byref(md), ctypes.byref(self._model.stage.desc),
                                                                 flags, ctypes.byref(h)), "rwkvb_engine_create_staged")
            else:
                native.check(self.lib.rwkvb_engine_create(ctypes.byref(md), flags, ctypes.byref(h)),
                             "rwkvb_engine_create")
            self._h = h
            att, wkv, ffn, logits = (ctypes.c_void_p() for _ in range(4))
            native.check(self.lib.rwkvb_engine_buffers(h, ctypes.byref(att), ctypes.byref(wkv), ctypes.byref(ffn),
                                                       ctypes.byref(logits)), "rwkvb_engine_buffers")
            L, C, H, N = s.n_layer, s.n_embd, s.n_head, s.head_size
            dev = self.device
            self.att_x = torch.as_tensor(_CudaArray(att.value, (L, C)), device=dev)
            self.wkv = torch.as_tensor(_CudaArray(wkv.value, (L, H, N, N)), device=dev)
            self.ffn_x = torch.as_tensor(_CudaArray(ffn.value, (L, C)), device=dev)
            self.logits = torch.as_tensor(_CudaArray(logits.value, (s.vocab,)), device=dev)
            n = ctypes.c_int32()
            native.check(self.lib.rwkvb_engine_launches_per_step(h, ctypes.byref(n)), "launches_per_step")
            self.launches_per_step = int(n.value)
            # 0: the whole decode loop runs as one persistent launch
            self.persistent_active = self.launches_per_step == 0

    # ------------------------------------------------------------ lifecycle
    def close(self) -> None:
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.device)
            self.lib.rwkvb_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self, stream=None) -> int:
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        return st.cuda_stream

    def _trace_raw(self) -> np.ndarray:
        cap = 4 * 65536
        buf = (ctypes.c_uint64 * cap)()
        n = ctypes.c_int32()
        native.check(self.lib.rwkvb_engine_trace(self._h, buf, cap, ctypes.byref(n)), "rwkvb_engine_trace")
        return np.frombuffer(buf, dtype=np.uint64, count=n.value).copy()

    def phase_trace(self) -> np.ndarray:
        """Phase timestamps of the last persistent launch, ``[2, 65536]`` ns
        (first CTA, last CTA); zeros where nothing was recorded."""
        return self._trace_raw()[: 2 * 65536].reshape(2, -1)

    def ring_trace(self) -> np.ndarray:
        """Ring events of the first CTA in the last persistent launch,
        ``[stages, 3]`` ns: producer issue, consumer wait end, consumer release."""
        raw = self._trace_raw()[2 * 65536:]
        n = len(raw) // 3
        return raw[: 3 * n].reshape(n, 3)

    # --------------------------------------------------------------- state
    def reset(self, stream=None) -> None:
        native.check(self.lib.rwkvb_engine_reset(self._h, self._stream(stream)), "rwkvb_engine_reset")

    def get_state(self) -> list[torch.Tensor]:
        """Clone of the state as ``RecurrentState.rwkv7_state`` (3 tensors per
        layer): three device copies, returned as per-layer views of them."""
        att, wkv, ffn = self.att_x.clone(), self.wkv.clone(), self.ffn_x.clone()
        out = []
        for i in range(self.shape.n_layer):
            out += [att[i], wkv[i], ffn[i]]
        return out

    def set_state(self, state: list[torch.Tensor]) -> None:
        if len(state) != 3 * self.shape.n_layer:
            raise ValueError(f"expected {3 * self.shape.n_layer} state tensors, got {len(state)}")
        for j, dst in enumerate((self.att_x, self.wkv, self.ffn_x)):
            parts = state[j::3]
            for i, t in enumerate(parts):
                if t.numel() != dst[i].numel():
                    raise ValueError(f"state tensor {3 * i + j} has {t.numel()} elements, expected {dst[i].numel()}")
            # one gather on the source device, one copy into the engine
            src = torch.stack([t.reshape(dst.shape[1:]) for t in parts])
            dst.copy_(src.to(self.device, torch.float32))

    # ------------------------------------------------------------- stepping
    def forward(self, tokens, stream=None) -> torch.Tensor:
        """Run one step per token; returns the device logits of the last step."""
        toks = (ctypes.c_int32 * len(tokens))(*[int(t) for t in tokens])
        native.check(self.lib.rwkvb_engine_forward(self._h, toks, len(tokens), self._stream(stream)),
                     "rwkvb_engine_forward")
        return self.logits

    def decode_greedy(self, first_token: int, n: int, stream=None) -> list[int]:
        out = (ctypes.c_int32 * max(n, 1))()
        native.check(self.lib.rwkvb_engine_decode_greedy(self._h, int(first_token), int(n), out,
                                                         self._stream(stream)), "rwkvb_engine_decode_greedy")
        return [int(v) for v in out[:n]]

    def decode_greedy_async(self, first_token: int, n: int, out: torch.Tensor, stream=None) -> None:
        if out.dtype != torch.int32 or not out.is_cuda or out.numel() < n:
            raise ValueError("out must be a CUDA int32 tensor with at least n elements")
        native.check(self.lib.rwkvb_engine_decode_greedy_async(self._h, int(first_token), int(n), out.data_ptr(),
                                                               self._stream(stream)),
                     "rwkvb_engine_decode_greedy_async")

    def _host_ring(self):
        ring = getattr(self, "_ring", None)
        if ring is None:
            ids, cnt, cancel, cap = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int32()
            native.check(self.lib.rwkvb_engine_host_ring(self._h, ctypes.byref(ids), ctypes.byref(cnt),
                                                         ctypes.byref(cancel), ctypes.byref(cap)),
                         "rwkvb_engine_host_ring")
            ring = (np.ctypeslib.as_array((ctypes.c_int32 * cap.value).from_address(ids.value)),
                    ctypes.c_uint32.from_address(cnt.value), ctypes.c_int32.from_address(cancel.value), cap.value)
            self._ring = ring
        return ring

    def decode_stream(self, first_token: int, n: int, on_token=None, should_stop=None, stream=None,
                      poll_s: float = 20e-6) -> list[int]:
        """Greedy decode of ``n`` steps (step 0 consumes ``first_token``) as ONE
        persistent launch whose ids reach the host through mapped pinned memory
        as the device makes them (``rwkvb_engine_decode_stream``).

        ``on_token(i, id)`` runs on this thread for every id in order;
        ``should_stop()`` is polled meanwhile.  When it returns true, or
        ``on_token`` raises, the device cancel word is set and the decode stops
        at a token boundary (the device acts on the word one token after it
        reads it, so no step waits on the bus); later ids are not passed to
        ``on_token``; the exception (if any) is re-raised after the launch has
        ended.  Returns the ids the device produced."""
        if not self.persistent_active:
            raise native.RwkvbError(native.RWKVB_EUNSUPPORTED, "decode_stream (persistent engines only)")
        ids_view, count, cancel, cap = self._host_ring()
        if n > cap:
            raise ValueError(f"n must be <= {cap}")
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        native.check(self.lib.rwkvb_engine_decode_stream(self._h, int(first_token), int(n), None, st.cuda_stream),
                     "rwkvb_engine_decode_stream")
        done = torch.cuda.Event()
        done.record(st)
        out: list[int] = []
        err: BaseException | None = None
        stopping = False
        while True:
            while len(out) < n:  # a slot holds -1 until its step's id replaces it
                tok = int(ids_view[len(out)])
                if tok < 0:
                    break
                out.append(tok)
                if on_token is not None and err is None and not stopping:
                    try:
                        on_token(len(out) - 1, tok)
                    except BaseException as e:  # noqa: BLE001 - re-raised below
                        err = e
                        cancel.value = 1
            if not stopping and err is None and should_stop is not None and should_stop():
                stopping = True
                cancel.value = 1
            if len(out) >= n:
                break
            if done.query():
                if min(int(count.value), n) <= len(out):
                    break
                continue
            time.sleep(poll_s)
        done.synchronize()
        native.check(self.lib.rwkvb_engine_check(self._h, st.cuda_stream), "rwkvb_engine_decode_stream")
        if err is not None:
            raise err
        return out

    def greedy(self, prompt: list[int], n_new: int, keep_logits: bool = False):
        """Prompt token by token, then ``n_new`` greedy ids (as the oracle's ``greedy``)."""
        rows = []
        if keep_logits:
            for t in prompt:
                self.forward([t])
                rows.append(self.logits.clone())
        else:
            self.forward(prompt)
        first = int(torch.argmax(self.logits).item())
        ids = [first]
        if keep_logits:
            for i in range(1, n_new):
                self.forward([ids[-1]])
                rows.append(self.logits.clone())
                ids.append(int(torch.argmax(self.logits).item()))
            return ids, torch.stack(rows)
        if n_new > 1:
            ids += self.decode_greedy(first, n_new - 1)
        return ids, None


class B200BatchEngine:
    """``batch`` (<= 64) independent sessions of one packed RWKV-7 model decoded
    together: one token step advances every session, with every projection a
    tcgen05 batched GEMM (``rwkvb_batch_*`` in the C ABI): integer GEMMs over
    digit rows for SG8 packs, fp16 GEMMs over decoded codebook tiles for LUT2
    packs (``lut2_tensor_cores=False``: fp32 CUDA-core products instead).

    The reference batches sessions with ``rwkv7_batch`` (ChatRWKV, not vendored)
    and otherwise loops sessions through ``forward_block_packed``; per session
    the result is that loop's, token for token.  State per layer and session
    keeps the ``RecurrentState.rwkv7_state`` triple."""

    def __init__(self, pack, batch: int, *, device: int | torch.device = 0, use_graph: bool = True,
                 pdl: bool = True, lut2_tensor_cores: bool = True):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("B200BatchEngine needs a CUDA device; there is no CPU path")
        self.lib = native.lib()
        self.batch = int(batch)
        with torch.cuda.device(self.device):
            self._model = pack if isinstance(pack, ModelUpload) else ModelUpload(pack, self.device)
            if self._model.stage is not None:
                raise ValueError("B200BatchEngine needs every layer resident (the model has streamed layers)")
            self.shape = s = self._model.shape
            flags = 0 if use_graph else native.FLAG_NO_GRAPH
            if not pdl:
                flags |= native.FLAG_NO_PDL
            if not lut2_tensor_cores:
                flags |= native.FLAG_LUT2_CUDA_CORES
            h = ctypes.c_void_p()
            native.check(self.lib.rwkvb_batch_create(ctypes.byref(self._model.md), self.batch, flags,
                                                     ctypes.byref(h)), "rwkvb_batch_create")
            self._h = h
            att, wkv, ffn, logits = (ctypes.c_void_p() for _ in range(4))
            native.check(self.lib.rwkvb_batch_buffers(h, ctypes.byref(att), ctypes.byref(wkv), ctypes.byref(ffn),
                                                      ctypes.byref(logits)), "rwkvb_batch_buffers")
            L, C, H, N, B = s.n_layer, s.n_embd, s.n_head, s.head_size, self.batch
            dev = self.device
            self.att_x = torch.as_tensor(_CudaArray(att.value, (L, B, C)), device=dev)
            self.wkv = torch.as_tensor(_CudaArray(wkv.value, (L, B, H, N, N)), device=dev)
            self.ffn_x = torch.as_tensor(_CudaArray(ffn.value, (L, B, C)), device=dev)
            self.logits = torch.as_tensor(_CudaArray(logits.value, (B, s.vocab)), device=dev)
            n = ctypes.c_int32()
            native.check(self.lib.rwkvb_batch_launches_per_step(h, ctypes.byref(n)), "launches_per_step")
            self.launches_per_step = int(n.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.device)
            self.lib.rwkvb_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self, stream=None) -> int:
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        return st.cuda_stream

    def reset(self, stream=None) -> None:
        native.check(self.lib.rwkvb_batch_reset(self._h, self._stream(stream)), "rwkvb_batch_reset")

    def forward(self, tokens, stream=None) -> torch.Tensor:
        """One step: session b consumes ``tokens[b]``; returns the device logits ``[batch, vocab]``."""
        if len(tokens) != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {len(tokens)}")
        toks = (ctypes.c_int32 * self.batch)(*[int(t) for t in tokens])
        native.check(self.lib.rwkvb_batch_forward(self._h, toks, self._stream(stream)), "rwkvb_batch_forward")
        return self.logits

    def prefill(self, prompts, stream=None) -> torch.Tensor:
        """Consume equal-length prompts (one per session) in order; returns the
        device logits ``[batch, vocab]`` of the last position.  Chunks of
        positions go through the tcgen05 GEMMs together (``rwkvb_batch_prefill``)."""
        if len(prompts) != self.batch or len({len(p) for p in prompts}) != 1:
            raise ValueError(f"expected {self.batch} prompts of equal length")
        n = len(prompts[0])
        toks = np.asarray(prompts, dtype=np.int32).reshape(-1)
        native.check(self.lib.rwkvb_batch_prefill(self._h, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n,
                                                  self._stream(stream)), "rwkvb_batch_prefill")
        return self.logits

    def decode_greedy(self, n: int, stream=None) -> np.ndarray:
        """``n`` greedy steps from the argmax of the current logits: ids ``[n, batch]``."""
        out = np.zeros((max(n, 1), self.batch), dtype=np.int32)
        native.check(self.lib.rwkvb_batch_decode_greedy(self._h, int(n),
                                                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                        self._stream(stream)), "rwkvb_batch_decode_greedy")
        return out[:n]

    def decode_greedy_async(self, n: int, out: torch.Tensor, stream=None) -> None:
        if out.dtype != torch.int32 or not out.is_cuda or out.numel() < n * self.batch:
            raise ValueError("out must be a CUDA int32 tensor with at least n * batch elements")
        native.check(self.lib.rwkvb_batch_decode_greedy_async(self._h, int(n), out.data_ptr(),
                                                              self._stream(stream)),
                     "rwkvb_batch_decode_greedy_async")

    def get_state(self, b: int) -> list[torch.Tensor]:
        """Clone of session ``b``'s state as ``RecurrentState.rwkv7_state`` (3 tensors per layer)."""
        out = []
        for i in range(self.shape.n_layer):
            out += [self.att_x[i, b].clone(), self.wkv[i, b].clone(), self.ffn_x[i, b].clone()]
        return out

    def set_state(self, b: int, state: list[torch.Tensor]) -> None:
        if len(state) != 3 * self.shape.n_layer:
            raise ValueError(f"expected {3 * self.shape.n_layer} state tensors, got {len(state)}")
        for i in range(self.shape.n_layer):
            self.att_x[i, b].copy_(state[3 * i].reshape(-1).to(self.device, torch.float32))
            self.wkv[i, b].copy_(state[3 * i + 1].reshape(self.wkv[i, b].shape).to(self.device, torch.float32))
            self.ffn_x[i, b].copy_(state[3 * i + 2].reshape(-1).to(self.device, torch.float32))
