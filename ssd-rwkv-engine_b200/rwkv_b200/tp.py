"""Tensor-parallel batched decode across the GPUs of one node (one process per
GPU, ``torch.distributed`` over NCCL for the plumbing).

The split is by attention heads, FFN rows and vocabulary rows (the layout the
C ABI's ``rwkvb_batch_create_tp`` documents):

=====================  =========================================  ==========
tensor                 shard held by rank r                       split
=====================  =========================================  ==========
att r/k/v weight       rows ``[c0, c1)`` (this rank's heads)       rows
att output weight      columns ``[c0, c1)``                        columns
att w2/a2/g2/v2        columns ``[c0, c1)``                        columns
att w0/a0/v0/k_k/k_a,  entries ``[c0, c1)``                        vector
ln_x weight/bias
att r_k ``[H, N]``     rows ``[h0, h1)``                           rows
ffn key weight         rows ``[f0, f1)``                           rows
ffn value weight       columns ``[f0, f1)``                        columns
head weight            rows ``[v0, v1)``                           rows
everything else        replicated (embedding, LayerNorms, mixes, adapter first stages)
=====================  =========================================  ==========

Per layer the output and FFN value projections produce partial sums that are
all-reduced; greedy decoding all-gathers each rank's (best logit, index) per
session and merges them first-maximum-wins, so every rank continues with the
same token ids.

SG8 blobs are sliced at the byte level: a slice whose element range starts on a
group boundary (rows), or whose column range is a whole number of groups
(columns), keeps every selected group's min/max record and codes unchanged, so
each rank dequantises exactly the values the full model holds
(``encode_scale_u8_grouped`` / ``decode_scale_u8_grouped`` in the reference's
``rwkv_ssd/format/quantize.py`` group the flattened row-major tensor).

The reference runs its 7.2B model on one device; this module is the multi-GPU
form of the same per-session computation (``packed_block_forward.py:76-166``
per layer, ``rwkv7_forward.py:791-809`` head, ``sampling.py:161-163`` argmax).
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import native
from .engine import ModelUpload, _CudaArray, infer_shape
from .synth import PackedTensor, RWKV7Shape

SG8_MAGIC = b"SG8\x01"

_ROWS_BY_CHANNEL = ("att.receptance.weight", "att.key.weight", "att.value.weight")
_COLS_BY_CHANNEL = ("att.output.weight", "att.w2", "att.a2", "att.g2", "att.v2")
_VEC_BY_CHANNEL = ("att.w0", "att.a0", "att.v0", "att.k_k", "att.k_a", "att.ln_x.weight", "att.ln_x.bias")


@dataclass(frozen=True)
class ShardPlan:
    """The slices rank ``rank`` of ``size`` holds."""

    rank: int
    size: int
    h0: int
    h1: int  # heads
    c0: int
    c1: int  # attention channels (= heads * head_size)
    f0: int
    f1: int  # FFN rows
    v0: int
    v1: int  # vocabulary rows

    @property
    def channels(self) -> int:
        return self.c1 - self.c0

    @property
    def vocab_local(self) -> int:
        return self.v1 - self.v0


def plan(shape: RWKV7Shape, rank: int, size: int) -> ShardPlan:
    """Shard plan of ``rank`` among ``size`` ranks.  Raises ``ValueError`` when
    the model does not split into the engine's 128-wide tiles: the heads must
    divide evenly with a multiple of 128 channels per rank, the FFN into
    128-multiples, and every vocabulary shard must be a multiple of 128 rows."""
    if size < 1 or not 0 <= rank < size:
        raise ValueError(f"bad rank {rank} of {size}")
    H, N, C, F, V = shape.n_head, shape.head_size, shape.n_embd, shape.ffn, shape.vocab
    if H % size or (H // size * N) % 128:
        raise ValueError(f"{H} heads of {N} do not split over {size} ranks in 128-channel shards")
    if F % (128 * size):
        raise ValueError(f"FFN width {F} does not split over {size} ranks in 128-row shards")
    hl = H // size
    fl = F // size
    vl = -(-V // (128 * size)) * 128
    v0, v1 = min(V, rank * vl), min(V, (rank + 1) * vl)
    if v1 - v0 <= 0 or (v1 - v0) % 128:
        raise ValueError(f"vocabulary {V} does not split over {size} ranks in 128-row shards")
    return ShardPlan(rank, size, rank * hl, (rank + 1) * hl, rank * hl * N, (rank + 1) * hl * N,
                     rank * fl, (rank + 1) * fl, v0, v1)


# --------------------------------------------------------------------------
# SG8 blob slicing
# --------------------------------------------------------------------------
def _as_u8(payload) -> torch.Tensor:
    if isinstance(payload, torch.Tensor):
        if payload.dtype != torch.uint8:
            raise TypeError("packed payload tensor must be uint8")
        return payload.reshape(-1)
    return torch.frombuffer(bytearray(payload), dtype=torch.uint8)


def _like(payload, t: torch.Tensor):
    return t.contiguous() if isinstance(payload, torch.Tensor) else t.numpy().tobytes()


def sg8_slice(payload, shape: tuple[int, int], rows: tuple[int, int] | None = None,
              cols: tuple[int, int] | None = None):
    """The SG8 blob of ``W[r0:r1, :]`` (``rows``) or ``W[:, c0:c1]`` (``cols``) of
    the ``shape`` matrix in ``payload`` (bytes, or a uint8 tensor on any
    device; the result has the same form).  The selected groups' records and
    codes are copied unchanged, so the slice dequantises bit-exactly to the
    same slice of the full matrix.  Raises ``ValueError`` for a slice that
    would cut a quantisation group."""
    if (rows is None) == (cols is None):
        raise ValueError("give exactly one of rows / cols")
    t = _as_u8(payload)
    head = bytes(t[:8].cpu().numpy().tobytes())
    if head[:4] != SG8_MAGIC:
        raise ValueError(f"not an SG8 blob (magic {head[:4]!r}); tensor parallelism needs SG8 matrices")
    (g,) = struct.unpack("<I", head[4:8])
    R, K = int(shape[0]), int(shape[1])
    n = R * K
    groups = -(-n // g)
    if t.numel() != 8 + 8 * groups + n:
        raise ValueError(f"SG8 blob of {t.numel()} bytes does not hold a {R}x{K} matrix in groups of {g}")
    recs = t[8:8 + 8 * groups]
    codes = t[8 + 8 * groups:]
    if rows is not None:
        r0, r1 = rows
        if not 0 <= r0 < r1 <= R:
            raise ValueError(f"row slice {rows} outside {R} rows")
        e0, e1 = r0 * K, r1 * K
        if e0 % g or (e1 % g and e1 != n):
            raise ValueError(f"row slice {rows} of a {R}x{K} matrix cuts a group of {g}")
        body = [recs[8 * (e0 // g):8 * (-(-e1 // g))], codes[e0:e1]]
    else:
        c0, c1 = cols
        if not 0 <= c0 < c1 <= K:
            raise ValueError(f"column slice {cols} outside {K} columns")
        if K % g or c0 % g or c1 % g:
            raise ValueError(f"column slice {cols} of a {R}x{K} matrix cuts a group of {g}")
        body = [recs.view(R, K // g, 8)[:, c0 // g:c1 // g].reshape(-1),
                codes.view(R, K)[:, c0:c1].reshape(-1)]
    out = torch.cat([t[:8]] + body)
    return _like(payload, out)


def _vec_slice(payload, lo: int, hi: int):
    if isinstance(payload, torch.Tensor):
        return payload.reshape(-1)[lo:hi].clone()
    return np.asarray(payload, dtype=np.float32).reshape(-1)[lo:hi].copy()


def shard_entry(name: str, e: PackedTensor, p: ShardPlan) -> PackedTensor:
    """Rank ``p.rank``'s part of one pack entry (replicated entries are returned as is)."""
    def mat(rows=None, cols=None):
        if e.codec != "sg8":
            raise ValueError(f"{name}: tensor parallelism needs SG8 matrices, got {e.codec}")
        R, K = e.shape
        shp = (rows[1] - rows[0], K) if rows else (R, cols[1] - cols[0])
        return PackedTensor(name, shp, "sg8", sg8_slice(e.payload, (R, K), rows=rows, cols=cols), dict(e.meta))

    if name == "head.weight":
        return mat(rows=(p.v0, p.v1))
    if not name.startswith("blocks."):
        return e
    if name.endswith(_ROWS_BY_CHANNEL):
        return mat(rows=(p.c0, p.c1))
    if name.endswith(_COLS_BY_CHANNEL):
        return mat(cols=(p.c0, p.c1))
    if name.endswith(".att.r_k"):
        return mat(rows=(p.h0, p.h1))
    if name.endswith(".ffn.key.weight"):
        return mat(rows=(p.f0, p.f1))
    if name.endswith(".ffn.value.weight"):
        return mat(cols=(p.f0, p.f1))
    if name.endswith(_VEC_BY_CHANNEL):
        shp = tuple(e.shape[:-1]) + (p.channels,)
        return PackedTensor(name, shp, e.codec, _vec_slice(e.payload, p.c0, p.c1), dict(e.meta))
    return e


def shard_pack(pack: dict[str, PackedTensor], rank: int, size: int) -> tuple[dict[str, PackedTensor], ShardPlan]:
    """Rank ``rank``'s shard of a full SG8 pack, with its plan."""
    p = plan(infer_shape(pack), rank, size)
    return {n: shard_entry(n, e, p) for n, e in pack.items()}, p


# --------------------------------------------------------------------------
# collectives
# --------------------------------------------------------------------------
class TPCollective:
    """The two collectives of the tensor-parallel step over a process group:
    kind 0 sums fp32 partial projections in place, kind 1 gathers each rank's
    per-session (best logit, index bits) pairs in rank order.  ``callback`` is
    what the C engine calls with device pointers; ``run`` works on tensors (the
    CPU tests drive it over ``gloo``)."""

    def __init__(self, group=None, device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = device
        self.error: BaseException | None = None
        self.calls = 0
        self._views: dict[tuple[int, int], torch.Tensor] = {}

    def warmup(self) -> None:
        """One collective outside any capture (creates the communicator)."""
        t = torch.zeros(1, device=self.device)
        dist.all_reduce(t, group=self.group)
        torch.cuda.synchronize(self.device)

    def agree(self, ok: bool) -> bool:
        """True on every rank when ``ok`` holds on every rank (eager, on the host's order)."""
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
        return bool(int(t.item()))

    def run(self, kind: int, send: torch.Tensor, recv: torch.Tensor) -> None:
        if kind == native.COLLECTIVE_ALLREDUCE_SUM_F32:
            if send.data_ptr() != recv.data_ptr():
                recv.copy_(send)
            dist.all_reduce(recv, op=dist.ReduceOp.SUM, group=self.group)
        elif kind == native.COLLECTIVE_ALLGATHER:
            dist.all_gather_into_tensor(recv, send, group=self.group)
        else:
            raise ValueError(f"unknown collective kind {kind}")
        self.calls += 1

    def _view(self, ptr: int, n: int) -> torch.Tensor:
        key = (ptr, n)
        t = self._views.get(key)
        if t is None:
            t = torch.as_tensor(_CudaArray(ptr, (n,), "<f4"), device=self.device)
            self._views[key] = t
        return t

    def callback(self, kind, send, recv, nbytes, stream, user) -> None:
        """C callback: issue the collective on ``stream``'s order.  Errors are
        kept in ``self.error`` (a ctypes callback cannot raise into C)."""
        try:
            n = int(nbytes) // 4
            s_t = self._view(int(send), n)
            r_t = s_t if recv == send else self._view(int(recv), n * (self.size if kind == 1 else 1))
            cur = torch.cuda.current_stream(self.device)
            if int(stream or 0) == int(cur.cuda_stream):
                self.run(kind, s_t, r_t)
            else:
                with torch.cuda.stream(torch.cuda.ExternalStream(int(stream), device=self.device)):
                    self.run(kind, s_t, r_t)
        except BaseException as e:  # noqa: BLE001 - reported by the engine call
            if self.error is None:
                self.error = e


class PeerExchange:
    """One exchange buffer per rank, mapped into every rank's process (CUDA IPC
    through the C ABI; the 64-byte handles travel through ``torch.distributed``).
    ``peers`` is the ``rwkvb_tp_desc.peer`` array: rank r's buffer as mapped
    here.  ``close`` is collective: every rank unmaps the others' buffers, then
    frees its own after the others are done with it."""

    def __init__(self, nbytes: int, group=None, device: torch.device | None = None):
        self.lib = native.lib()
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        native.check(self.lib.rwkvb_ipc_alloc(int(nbytes), ctypes.byref(own), handle), "rwkvb_ipc_alloc")
        self._own = own
        mine = torch.tensor(list(handle.raw), dtype=torch.uint8, device=self.device)
        allh = torch.empty(self.size * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        raw = bytes(allh.cpu().numpy().tolist())
        self._opened: list[ctypes.c_void_p] = []
        self.peers = (ctypes.c_void_p * self.size)()
        for r in range(self.size):
            if r == self.rank:
                self.peers[r] = own.value
                continue
            ptr = ctypes.c_void_p()
            native.check(self.lib.rwkvb_ipc_open(raw[64 * r:64 * (r + 1)], ctypes.byref(ptr)), "rwkvb_ipc_open")
            self._opened.append(ptr)
            self.peers[r] = ptr.value

    def close(self) -> None:
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every rank's kernels are done with every buffer
        for ptr in self._opened:
            self.lib.rwkvb_ipc_close(ptr)
        self._opened = []
        dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        self.lib.rwkvb_ipc_free(self._own)
        self._own = None


# --------------------------------------------------------------------------
# engine
# --------------------------------------------------------------------------
class B200TPBatchEngine:
    """``batch`` (<= 64) sessions of one SG8 RWKV-7 model decoded with the model
    split over the ranks of ``group`` (every rank constructs it with the same
    full pack, or with its own shard and ``plan``, and calls the same methods
    with the same arguments; ``exchange="p2p"`` runs the all-reduces and the
    argmax gather in the engine's own kernels over NVLink peer memory instead of
    NCCL through the host callback).  Logits are this rank's vocabulary rows
    ``[plan.v0, plan.v1)``; ``logits_full`` gathers them.  Greedy ids are the
    same on every rank."""

    def __init__(self, pack, batch: int, *, group=None, device: torch.device | None = None,
                 use_graph: bool = False, shard_plan: ShardPlan | None = None, collective: TPCollective | None = None,
                 exchange: str = "nccl"):
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("B200TPBatchEngine needs a CUDA device; there is no CPU path")
        if collective is None:
            if not (dist.is_available() and dist.is_initialized()):
                raise RuntimeError("B200TPBatchEngine needs an initialised torch.distributed process group")
            collective = TPCollective(group, self.device)
        self._coll = collective
        self.group = group
        self.rank = collective.rank
        self.size = collective.size
        if self.size < 2:
            raise ValueError("tensor parallelism needs at least 2 ranks")
        if shard_plan is None:
            local, shard_plan = shard_pack(pack, self.rank, self.size)
        else:
            local = pack
        if shard_plan.rank != self.rank or shard_plan.size != self.size:
            raise ValueError("shard plan does not match this rank")
        self.plan = shard_plan
        self.lib = native.lib()
        self.batch = int(batch)
        with torch.cuda.device(self.device):
            self._model = ModelUpload(local, self.device)
            s = self._model.shape
            self.shape = s
            self._coll.warmup()
            self._cfn = native.COLLECTIVE_FN(self._coll.callback)
            desc = native.TPDesc(self.rank, self.size, shard_plan.v0, self._cfn, None, None)
            self.exchange = exchange
            self._x = None
            if exchange == "p2p":
                # the all-reduces and the argmax gather run in the engine's own
                # kernels over peer memory (no host callback, no NCCL)
                nbytes = ctypes.c_uint64()
                native.check(self.lib.rwkvb_batch_tp_exchange_bytes(ctypes.byref(self._model.md), self.batch,
                                                                    ctypes.byref(nbytes)),
                             "rwkvb_batch_tp_exchange_bytes")
                self._x = PeerExchange(int(nbytes.value), group, self.device)
                desc.peer = self._x.peers
            elif exchange != "nccl":
                raise ValueError(f"exchange must be 'nccl' or 'p2p', not {exchange!r}")
            h = ctypes.c_void_p()
            flags = 0 if use_graph else native.FLAG_NO_GRAPH
            native.check(self.lib.rwkvb_batch_create_tp(ctypes.byref(self._model.md), self.batch,
                                                        ctypes.byref(desc), flags, ctypes.byref(h)),
                         "rwkvb_batch_create_tp")
            self._h = h
            self.use_graph = bool(use_graph)
            if self.use_graph:
                # capture the step (collectives included) on every rank, then
                # agree that all captures succeeded before any rank launches one
                st = self.lib.rwkvb_batch_prepare(h, self._stream())
                err, self._coll.error = self._coll.error, None
                ok = self._coll.agree(st == native.RWKVB_OK and err is None)
                if not ok:
                    self.lib.rwkvb_batch_destroy(h)
                    self._h = None
                    if err is not None:
                        raise RuntimeError("capturing the tensor-parallel step failed") from err
                    native.check(st if st != native.RWKVB_OK else native.RWKVB_ECUDA,
                                 "rwkvb_batch_prepare (on some rank)")
            att, wkv, ffn, logits = (ctypes.c_void_p() for _ in range(4))
            native.check(self.lib.rwkvb_batch_buffers(h, ctypes.byref(att), ctypes.byref(wkv), ctypes.byref(ffn),
                                                      ctypes.byref(logits)), "rwkvb_batch_buffers")
            L, C, N, B = s.n_layer, s.n_embd, s.head_size, self.batch
            hl = shard_plan.h1 - shard_plan.h0
            dev = self.device
            self.att_x = torch.as_tensor(_CudaArray(att.value, (L, B, C)), device=dev)
            self.wkv = torch.as_tensor(_CudaArray(wkv.value, (L, B, hl, N, N)), device=dev)
            self.ffn_x = torch.as_tensor(_CudaArray(ffn.value, (L, B, C)), device=dev)
            self.logits = torch.as_tensor(_CudaArray(logits.value, (B, shard_plan.vocab_local)), device=dev)
            n = ctypes.c_int32()
            native.check(self.lib.rwkvb_batch_launches_per_step(h, ctypes.byref(n)), "launches_per_step")
            self.launches_per_step = int(n.value)

    def _checked(self, status: int, what: str) -> None:
        err, self._coll.error = self._coll.error, None
        if err is not None:
            raise RuntimeError(f"{what}: collective failed") from err
        native.check(status, what)

    def close(self) -> None:
        """Release the engine; collective when the peer exchange is in use."""
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.device)
            self.lib.rwkvb_batch_destroy(self._h)
            self._h = None
        if getattr(self, "_x", None) is not None:
            self._x.close()
            self._x = None

    def __del__(self):
        # not collective: release the engine only (the exchange buffers are
        # released by close(), which every rank calls, or at process exit)
        try:
            if getattr(self, "_h", None):
                self.lib.rwkvb_batch_destroy(self._h)
                self._h = None
        except Exception:
            pass

    def _stream(self, stream=None) -> int:
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        return st.cuda_stream

    @property
    def collective_calls(self) -> int:
        return self._coll.calls

    def reset(self, stream=None) -> None:
        native.check(self.lib.rwkvb_batch_reset(self._h, self._stream(stream)), "rwkvb_batch_reset")

    def forward(self, tokens, stream=None) -> torch.Tensor:
        """One step: session b consumes ``tokens[b]`` (the same ids on every
        rank); returns this rank's logits ``[batch, vocab_local]``."""
        if len(tokens) != self.batch:
            raise ValueError(f"expected {self.batch} tokens, got {len(tokens)}")
        toks = (ctypes.c_int32 * self.batch)(*[int(t) for t in tokens])
        with torch.cuda.device(self.device):
            self._checked(self.lib.rwkvb_batch_forward(self._h, toks, self._stream(stream)), "rwkvb_batch_forward")
        return self.logits

    def prefill(self, prompts, stream=None) -> torch.Tensor:
        """Consume equal-length prompts position by position (tensor-parallel
        decode steps)."""
        if len(prompts) != self.batch or len({len(p) for p in prompts}) != 1:
            raise ValueError(f"expected {self.batch} prompts of equal length")
        for pos in range(len(prompts[0])):
            self.forward([p[pos] for p in prompts], stream)
        return self.logits

    def decode_greedy(self, n: int, stream=None) -> np.ndarray:
        """``n`` greedy steps from the argmax of the current (global) logits: ids ``[n, batch]``."""
        out = np.zeros((max(n, 1), self.batch), dtype=np.int32)
        with torch.cuda.device(self.device):
            self._checked(self.lib.rwkvb_batch_decode_greedy(self._h, int(n),
                                                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                             self._stream(stream)), "rwkvb_batch_decode_greedy")
        return out[:n]

    def decode_greedy_async(self, n: int, out: torch.Tensor, stream=None) -> None:
        if out.dtype != torch.int32 or not out.is_cuda or out.numel() < n * self.batch:
            raise ValueError("out must be a CUDA int32 tensor with at least n * batch elements")
        with torch.cuda.device(self.device):
            self._checked(self.lib.rwkvb_batch_decode_greedy_async(self._h, int(n), out.data_ptr(),
                                                                   self._stream(stream)),
                          "rwkvb_batch_decode_greedy_async")

    def logits_full(self) -> torch.Tensor:
        """All ranks' logits ``[batch, vocab]`` (a collective: every rank calls it)."""
        vl = self.plan.vocab_local
        cap = -(-self.shape.vocab // (128 * self.size)) * 128
        loc = torch.zeros((self.batch, cap), dtype=torch.float32, device=self.device)
        loc[:, :vl].copy_(self.logits)
        parts = torch.empty((self.size, self.batch, cap), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            self._coll.run(native.COLLECTIVE_ALLGATHER, loc.reshape(-1), parts.reshape(-1))
        self._coll.calls -= 1  # not a step collective
        return parts.permute(1, 0, 2).reshape(self.batch, -1)[:, :self.shape.vocab]
