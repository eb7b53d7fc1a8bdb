"""Host side of the tensor-parallel decode (``rwkv_b200.tp``) on the CPU: shard
plans, byte-level SG8 slicing (bit-exact against the oracle decode), shard
packs that reassemble the full model, and a two-rank ``gloo`` run of the oracle
forward over the shards (partial output / FFN value sums all-reduced, argmax
bests all-gathered and merged first-maximum-wins) against the single-device
oracle."""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import codec as oc
from oracle.forward import OracleRWKV7
from rwkv_b200 import native, synth, tp


def _blob(w: np.ndarray, g: int = 128) -> bytes:
    return oc.encode_sg8(w.reshape(-1).astype(np.float32), g)


@pytest.mark.parametrize("R,K", [(6, 256), (9, 64), (10, 64), (4, 384)])
def test_sg8_row_slices_are_bit_exact(R, K):
    w = np.random.default_rng(R * K).standard_normal((R, K)).astype(np.float32)
    blob = _blob(w)
    full = oc.decode_sg8(blob, R * K).reshape(R, K)
    ok = 0
    for r0 in range(R):
        for r1 in range(r0 + 1, R + 1):
            e0, e1 = r0 * K, r1 * K
            if e0 % 128 or (e1 % 128 and e1 != R * K):
                with pytest.raises(ValueError):
                    tp.sg8_slice(blob, (R, K), rows=(r0, r1))
                continue
            part = tp.sg8_slice(blob, (R, K), rows=(r0, r1))
            assert isinstance(part, bytes)
            got = oc.decode_sg8(part, (r1 - r0) * K).reshape(r1 - r0, K)
            assert np.array_equal(got.view(np.uint32), full[r0:r1].view(np.uint32))
            t = tp.sg8_slice(torch.frombuffer(bytearray(blob), dtype=torch.uint8), (R, K), rows=(r0, r1))
            assert t.numpy().tobytes() == part
            ok += 1
    assert ok > 0


def test_sg8_column_slices_are_bit_exact():
    R, K = 5, 512
    w = np.random.default_rng(11).standard_normal((R, K)).astype(np.float32)
    blob = _blob(w)
    full = oc.decode_sg8(blob, R * K).reshape(R, K)
    for c0, c1 in [(0, 128), (128, 384), (256, 512), (0, 512)]:
        part = tp.sg8_slice(blob, (R, K), cols=(c0, c1))
        got = oc.decode_sg8(part, R * (c1 - c0)).reshape(R, c1 - c0)
        assert np.array_equal(got.view(np.uint32), full[:, c0:c1].view(np.uint32))
    for bad in [(64, 192), (0, 100), (128, 600)]:
        with pytest.raises(ValueError):
            tp.sg8_slice(blob, (R, K), cols=bad)
    with pytest.raises(ValueError):
        tp.sg8_slice(blob, (R, K))
    with pytest.raises(ValueError):
        tp.sg8_slice(b"TR2\x04" + blob[4:], (R, K), rows=(0, 1))


def test_plans():
    P = synth.PRESETS
    for size in (2, 4, 8):
        plans = [tp.plan(P["7.2b"], r, size) for r in range(size)]
        assert [p.c0 for p in plans] == [r * 4096 // size for r in range(size)]
        assert plans[-1].c1 == 4096 and plans[-1].f1 == 16384 and plans[-1].v1 == 65536
        assert all(p.channels % 128 == 0 and p.vocab_local % 128 == 0 for p in plans)
    assert tp.plan(P["2.9b"], 3, 4).c0 == 1920
    with pytest.raises(ValueError):
        tp.plan(P["2.9b"], 0, 8)  # 5 heads per rank: 320 channels
    with pytest.raises(ValueError):
        tp.plan(P["tiny"], 0, 4)  # 1 head per rank
    with pytest.raises(ValueError):
        tp.plan(P["tiny"], 2, 2)
    odd = synth.RWKV7Shape(2, 256, 64, 1024, 1920, 32, 32, 32, 64)
    assert [(p.v0, p.v1) for p in (tp.plan(odd, r, 2) for r in range(2))] == [(0, 1024), (1024, 1920)]


# shapes of the rank tests: the tiny preset (4 heads: 2 ranks at most) and
# 2-layer models of 8 and 16 heads, so that 4 and 8 ranks hold 128 channels each
SHAPES = {"tiny": synth.PRESETS["tiny"], "wide8h": synth.RWKV7Shape(2, 512, 64, 2048, 1024, 32, 32, 32, 64),
          "wide16h": synth.RWKV7Shape(2, 1024, 64, 4096, 1024, 32, 32, 32, 64)}


def _pack(key: str, seed: int):
    shape = SHAPES[key]
    return shape, synth.make_pack(synth.generate_state_dict(shape, seed, "cpu"), policy="sg8")


def _tiny_pack(seed: int):
    return _pack("tiny", seed)


def test_shards_reassemble_the_full_pack():
    shape, pack = _tiny_pack(3)
    shards = [tp.shard_pack(pack, r, 2) for r in range(2)]
    for name, e in pack.items():
        parts = [s[name] for s, _ in shards]
        if all(p is e for p in parts):
            continue  # replicated
        if e.codec == "none":
            got = np.concatenate([np.asarray(p.payload).reshape(-1) for p in parts])
            assert np.array_equal(got, np.asarray(e.payload).reshape(-1)), name
            continue
        R, K = e.shape
        full = oc.decode_sg8(e.payload, R * K).reshape(R, K)
        dec = [oc.decode_sg8(p.payload, p.shape[0] * p.shape[1]).reshape(p.shape) for p in parts]
        axis = 0 if parts[0].shape[1] == K else 1
        assert np.array_equal(np.concatenate(dec, axis=axis).view(np.uint32), full.view(np.uint32)), name
    # what is split, and how
    p0 = shards[0][0]
    assert p0["blocks.1.att.receptance.weight"].shape == (128, 256)
    assert p0["blocks.1.att.output.weight"].shape == (256, 128)
    assert p0["blocks.1.att.w2"].shape == (32, 128)
    assert p0["blocks.1.att.w1"] is pack["blocks.1.att.w1"]
    assert p0["blocks.1.att.r_k"].shape == (2, 64)
    assert p0["blocks.1.ffn.key.weight"].shape == (512, 256)
    assert p0["blocks.1.ffn.value.weight"].shape == (256, 512)
    assert p0["head.weight"].shape == (512, 256)
    assert p0["emb.weight"] is pack["emb.weight"]
    assert p0["blocks.1.att.k_k"].shape == (1, 1, 128)


# ------------------------------------------------------------ two gloo ranks
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _global_argmax(coll: tp.TPCollective, logits: np.ndarray, v0: int) -> int:
    """Each rank's (first max, index) pair all-gathered, merged first-maximum-wins
    in rank order (the rule of the device merge)."""
    i = int(np.argmax(logits))
    mine = torch.tensor([float(logits[i]), 0.0], dtype=torch.float32)
    mine[1:].view(torch.int32)[0] = v0 + i
    allp = torch.empty(2 * coll.size, dtype=torch.float32)
    coll.run(native.COLLECTIVE_ALLGATHER, mine, allp)
    best, bi = -np.inf, None
    for r in range(coll.size):
        val = float(allp[2 * r])
        idx = int(allp[2 * r + 1:2 * r + 2].view(torch.int32)[0])
        if val > best or (val == best and idx < bi):
            best, bi = val, idx
    return bi


def _worker(rank: int, world: int, port: int, q, key: str = "tiny") -> None:
    sys.path[:0] = [p for p in os.environ.get("RWKVB_TEST_PATH", "").split(os.pathsep) if p]
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        shape, pack = _pack(key, 5)
        local, plan = tp.shard_pack(pack, rank, world)
        coll = tp.TPCollective()

        def reduce(v: np.ndarray) -> np.ndarray:
            t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
            coll.run(native.COLLECTIVE_ALLREDUCE_SUM_F32, t, t)
            return t.numpy()

        oracle = OracleRWKV7(local, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size,
                             reduce=reduce, argmax=lambda lg: _global_argmax(coll, lg, plan.v0))
        prompt = synth.seeded_prompt(6, shape.vocab, 5)
        ids, logits, state = oracle.greedy(prompt, 5)
        q.put((rank, plan, ids, logits, state, coll.calls))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put(("error", rank, repr(e)))


def _ranks_match_single_device(world: int, key: str) -> None:
    """`world` gloo ranks run the oracle over their shards (all-reduce and
    argmax hooks); ids, logits and state must equal the single-device oracle."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["RWKVB_TEST_PATH"] = os.pathsep.join(sys.path)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, key)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert not any(o[0] == "error" for o in out), out
    by_rank = {o[0]: o for o in out}
    shape, pack = _pack(key, 5)
    ref = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    prompt = synth.seeded_prompt(6, shape.vocab, 5)
    ids_ref, logits_ref, state_ref = ref.greedy(prompt, 5)
    logits = np.concatenate([by_rank[r][3] for r in range(world)], axis=1)
    for r in range(world):
        _, plan, ids, _, state, calls = by_rank[r]
        assert ids == ids_ref
        # per forward: 2 all-reduces per layer; per greedy pick: one all-gather
        assert calls == (6 + 4) * 2 * shape.n_layer + 5
        for layer in range(shape.n_layer):
            np.testing.assert_allclose(state[3 * layer], state_ref[3 * layer], rtol=0, atol=1e-4)
            np.testing.assert_allclose(state[3 * layer + 1], state_ref[3 * layer + 1][plan.h0:plan.h1],
                                       rtol=0, atol=1e-4)
            np.testing.assert_allclose(state[3 * layer + 2], state_ref[3 * layer + 2], rtol=0, atol=1e-4)
    np.testing.assert_allclose(logits, logits_ref, rtol=0, atol=1e-4)


def test_two_rank_oracle_over_shards_matches_single_device():
    _ranks_match_single_device(2, "tiny")


def test_four_rank_oracle_over_shards_matches_single_device():
    _ranks_match_single_device(4, "wide8h")


def test_eight_rank_oracle_over_shards_matches_single_device():
    _ranks_match_single_device(8, "wide16h")


# ------------------------------------------------ peer-exchange host side
def _peer_worker(rank: int, world: int, port: int, q) -> None:
    """PeerExchange over gloo with a fake of the C ABI's IPC calls: rank r's
    "handle" is 64 bytes of (r + 1), its own buffer 0x10000 (r + 1), and opening
    rank s's handle maps it at 0x7000000 + 0x10000 (s + 1)."""
    sys.path[:0] = [p for p in os.environ.get("RWKVB_TEST_PATH", "").split(os.pathsep) if p]
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        opened, closed, freed = [], [], []

        class FakeIpc:
            def rwkvb_ipc_alloc(self, nbytes, own_ref, handle):
                own_ref._obj.value = 0x10000 * (rank + 1)
                ctypes.memmove(handle, bytes([rank + 1]) * 64, 64)
                return native.RWKVB_OK

            def rwkvb_ipc_open(self, raw, ptr_ref):
                src = raw[0] - 1
                if raw != bytes([src + 1]) * 64 or src == rank:
                    return native.RWKVB_EARG
                ptr_ref._obj.value = 0x7000000 + 0x10000 * (src + 1)
                opened.append(src)
                return native.RWKVB_OK

            def rwkvb_ipc_close(self, ptr):
                closed.append(ptr.value)
                return native.RWKVB_OK

            def rwkvb_ipc_free(self, ptr):
                freed.append(ptr.value)
                return native.RWKVB_OK

        native.lib = lambda: FakeIpc()
        torch.cuda.synchronize = lambda *a, **k: None  # no device work to wait for on the CPU
        ex = tp.PeerExchange(4096, device=torch.device("cpu"))
        peers = [int(ex.peers[r]) for r in range(world)]
        ex.close()
        ex.close()  # a second close is a no-op
        q.put((rank, peers, opened, closed, freed))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put(("error", rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_maps_every_rank_in_rank_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["RWKVB_TEST_PATH"] = os.pathsep.join(sys.path)
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert not any(o[0] == "error" for o in out), out
    for rank, peers, opened, closed, freed in out:
        want = [0x10000 * (r + 1) if r == rank else 0x7000000 + 0x10000 * (r + 1) for r in range(world)]
        assert peers == want
        assert opened == [r for r in range(world) if r != rank]
        assert closed == [want[r] for r in range(world) if r != rank]
        assert freed == [0x10000 * (rank + 1)]
