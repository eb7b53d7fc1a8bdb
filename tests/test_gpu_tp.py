"""GPU parity of the tensor-parallel batched decode (``rwkvb_batch_create_tp``
through ``rwkv_b200.tp.B200TPBatchEngine``) on two GPUs, one process each over
NCCL: greedy ids identical to the single-GPU batched engine, gathered logits and
the replicated / head-sharded state within 1e-3 max-abs (partial sums are
all-reduced, so the summation order differs from one GPU's)."""

from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)
import threading  # noqa: E402

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from rwkv_b200 import synth, tp  # noqa: E402

TOL = 1e-3
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


class _ThreadGroup:
    """Shared slots of ranks emulated as threads of one process on one GPU."""

    def __init__(self, size: int):
        self.size = size
        self.bar = threading.Barrier(size, timeout=120)
        self.send = [None] * size
        self.ev_a = [None] * size
        self.ev_b = [None] * size


class _ThreadRankCollective(tp.TPCollective):
    """The step collectives between thread-ranks: every rank waits (on the
    device, through events) for all ranks' inputs, forms the same rank-ordered
    sum / concatenation, and writes it only after every rank has read the
    inputs.  No kernel waits on another; the host threads meet at barriers."""

    def __init__(self, grp: _ThreadGroup, rank: int, device: torch.device):
        self.group = None
        self.rank, self.size, self.device = rank, grp.size, device
        self.error = None
        self.calls = 0
        self._views = {}
        self.grp = grp

    def warmup(self) -> None:
        pass

    def agree(self, ok: bool) -> bool:
        return ok

    def run(self, kind, send, recv):
        g, st = self.grp, torch.cuda.current_stream(self.device)
        ev = torch.cuda.Event()
        ev.record(st)
        g.send[self.rank], g.ev_a[self.rank] = send, ev
        g.bar.wait()
        for r in range(self.size):
            if r != self.rank:
                st.wait_event(g.ev_a[r])
        if kind == 0:
            out = g.send[0].clone()
            for r in range(1, self.size):
                out += g.send[r]
        else:
            out = torch.cat([g.send[r] for r in range(self.size)])
        ev = torch.cuda.Event()
        ev.record(st)
        g.ev_b[self.rank] = ev
        g.bar.wait()
        for r in range(self.size):
            if r != self.rank:
                st.wait_event(g.ev_b[r])
        recv.copy_(out)
        g.bar.wait()
        self.calls += 1


def _threads(fns, grp: _ThreadGroup):
    errs, out = [], [None] * len(fns)

    def body(i):
        try:
            torch.cuda.set_device(0)
            with torch.cuda.stream(torch.cuda.Stream()):
                out[i] = fns[i]()
                torch.cuda.current_stream().synchronize()
        except BaseException as e:  # noqa: BLE001
            import traceback
            errs.append(traceback.format_exc())
            grp.bar.abort()  # release the other ranks from their barrier
    th = [threading.Thread(target=body, args=(i,)) for i in range(len(fns))]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=600)
    assert not errs, errs
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_pack(preset: str, seed: int, rank: int, world: int):
    from rwkv_b200 import tp
    shape = synth.PRESETS[preset]
    p = tp.plan(shape, rank, world)
    local = synth.make_pack_streaming(shape, seed, "cuda", policy="sg8",
                                      transform=lambda n, e: tp.shard_entry(n, e, p))
    return shape, local, p


def _worker(rank: int, world: int, port: int, case: dict, q) -> None:
    sys.path[:0] = [p for p in os.environ.get("RWKVB_TEST_PATH", "").split(os.pathsep) if p]
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
        from rwkv_b200.tp import B200TPBatchEngine
        shape, local, plan = _make_pack(case["preset"], case["seed"], rank, world)
        nb, length, n_new = case["nb"], case["length"], case["n_new"]
        prompts = [synth.seeded_prompt(length, shape.vocab, case["seed"] + 101 * b) for b in range(nb)]
        eng = B200TPBatchEngine(local, nb, shard_plan=plan, use_graph=case.get("graph", False),
                                exchange=case.get("exchange", "nccl"))
        try:
            eng.prefill(prompts)
            first = eng.logits_full().argmax(dim=1).cpu().numpy()
            ids = eng.decode_greedy(n_new)
            logits = eng.logits_full().cpu().numpy()
            res = dict(first=first, ids=ids, logits=logits, att_x=eng.att_x.cpu().numpy(),
                       ffn_x=eng.ffn_x.cpu().numpy(), wkv=eng.wkv.cpu().numpy(), h0=plan.h0, h1=plan.h1,
                       calls=eng.collective_calls, launches=eng.launches_per_step)
        finally:
            eng.close()
        q.put((rank, res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        import traceback
        q.put(("error", rank, traceback.format_exc() + repr(e)))


def _run_tp(case: dict, world: int = 2) -> dict:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    os.environ["RWKVB_TEST_PATH"] = os.pathsep.join(sys.path)
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in range(world):
            out.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():  # pragma: no cover
                p.kill()
    errs = [o for o in out if o[0] == "error"]
    assert not errs, errs
    return {r: res for r, res in out}


def _prompts(case: dict) -> list[list[int]]:
    shape = synth.PRESETS[case["preset"]]
    return [synth.seeded_prompt(case["length"], shape.vocab, case["seed"] + 101 * b) for b in range(case["nb"])]


def _single(case: dict, prompts=None) -> dict:
    from rwkv_b200.engine import B200BatchEngine
    shape = synth.PRESETS[case["preset"]]
    pack = synth.make_pack_streaming(shape, case["seed"], "cuda", policy="sg8")
    nb, n_new = case["nb"], case["n_new"]
    prompts = prompts if prompts is not None else _prompts(case)
    length = len(prompts[0])
    eng = B200BatchEngine(pack, nb)
    try:
        for pos in range(length):
            eng.forward([p[pos] for p in prompts])
        first = eng.logits.argmax(dim=1).cpu().numpy()
        ids = eng.decode_greedy(n_new)
        return dict(first=first, ids=ids, logits=eng.logits.cpu().numpy(), att_x=eng.att_x.cpu().numpy(),
                    ffn_x=eng.ffn_x.cpu().numpy(), wkv=eng.wkv.cpu().numpy())
    finally:
        eng.close()
        del pack
        torch.cuda.empty_cache()


def _first_divergence(got: dict, ref: dict, n_layer: int) -> str:
    for l in range(n_layer):
        for key in ("att_x", "wkv", "ffn_x"):
            a = got[key][l]
            b = ref[key][l] if key != "wkv" else ref[key][l][:, got["h0"]:got["h1"]]
            d = float(np.abs(a - b).max())
            if d > TOL:
                return f"layer {l} {key}: max abs diff {d:.3g}"
    d = float(np.abs(got["logits"] - ref["logits"]).max())
    return f"logits: max abs diff {d:.3g}"


CASES = [dict(preset="tiny", seed=31, nb=5, length=6, n_new=8),
         dict(preset="7.2b-l4", seed=37, nb=8, length=3, n_new=3)]


@pytest.mark.parametrize("case", CASES, ids=["tiny", "7.2b-l4"])
def test_tp2_as_threads_on_one_gpu_matches_single_engine(case):
    """Two tensor-parallel ranks as two threads on GPU 0 (the collectives are
    event-ordered device sums instead of NCCL): the sharded engine path itself."""
    shape = synth.PRESETS[case["preset"]]
    nb, length, n_new = case["nb"], case["length"], case["n_new"]
    prompts = _prompts(case)
    dev = torch.device("cuda", 0)
    grp = _ThreadGroup(2)
    engines = []
    for r in range(2):
        p = tp.plan(shape, r, 2)
        local = synth.make_pack_streaming(shape, case["seed"], "cuda", policy="sg8",
                                          transform=lambda n, e, p=p: tp.shard_entry(n, e, p))
        engines.append(tp.B200TPBatchEngine(local, nb, device=dev, shard_plan=p,
                                            collective=_ThreadRankCollective(grp, r, dev)))
        del local
    try:
        def one_step(r):
            return lambda: engines[r].forward([p[0] for p in prompts])
        _threads([one_step(0), one_step(1)], grp)
        step1 = [dict(att_x=e.att_x.cpu().numpy(), wkv=e.wkv.cpu().numpy(), ffn_x=e.ffn_x.cpu().numpy(),
                      h0=e.plan.h0, h1=e.plan.h1) for e in engines]

        def rest(r):
            def f():
                e = engines[r]
                for pos in range(1, length):
                    e.forward([p[pos] for p in prompts])
                ids = e.decode_greedy(n_new)
                return ids
            return f
        ids = _threads([rest(0), rest(1)], grp)
        full = _threads([lambda: engines[0].logits_full(), lambda: engines[1].logits_full()], grp)
        got = [dict(ids=ids[r], logits=full[r].cpu().numpy(), att_x=engines[r].att_x.cpu().numpy(),
                    ffn_x=engines[r].ffn_x.cpu().numpy(), wkv=engines[r].wkv.cpu().numpy(),
                    h0=engines[r].plan.h0, h1=engines[r].plan.h1) for r in range(2)]
    finally:
        for e in engines:
            e.close()
    ref1 = _single(dict(case, n_new=0), [p[:1] for p in prompts])
    ref = _single(case)
    for r in range(2):
        msg = _first_divergence(dict(step1[r], logits=ref1["logits"]), ref1, shape.n_layer)
        assert msg.startswith("logits"), f"rank {r}, first step: {msg}"
        assert np.array_equal(got[r]["ids"], ref["ids"]), (r, _first_divergence(got[r], ref, shape.n_layer))
        np.testing.assert_allclose(got[r]["logits"], ref["logits"], rtol=0, atol=TOL)
        assert _first_divergence(got[r], ref, shape.n_layer).startswith("logits")


@two_gpus
@pytest.mark.parametrize("case", CASES + [dict(c, graph=True) for c in CASES]
                         + [dict(c, exchange="p2p") for c in CASES] + [dict(c, graph=True, exchange="p2p") for c in CASES],
                         ids=["tiny", "7.2b-l4", "tiny-graph", "7.2b-l4-graph", "tiny-p2p", "7.2b-l4-p2p",
                              "tiny-p2p-graph", "7.2b-l4-p2p-graph"])
def test_tp2_matches_single_gpu_batched_engine(case):
    got = _run_tp(case)
    ref = _single(case)
    shape = synth.PRESETS[case["preset"]]
    for r, res in got.items():
        assert np.array_equal(res["first"], ref["first"]), r
        assert np.array_equal(res["ids"], ref["ids"]), r
        np.testing.assert_allclose(res["logits"], ref["logits"], rtol=0, atol=TOL)
        np.testing.assert_allclose(res["att_x"], ref["att_x"], rtol=0, atol=TOL)
        np.testing.assert_allclose(res["ffn_x"], ref["ffn_x"], rtol=0, atol=TOL)
        np.testing.assert_allclose(res["wkv"], ref["wkv"][:, :, res["h0"]:res["h1"]], rtol=0, atol=TOL)
        # two all-reduces per layer and one all-gather per step (logits_full's
        # gathers are not counted); a CUDA graph issues them once, at capture
        steps = 1 if case.get("graph") else case["length"] + case["n_new"]
        # the peer exchange does not call back at all
        expect = 0 if case.get("exchange") == "p2p" else steps * (2 * shape.n_layer + 1)
        assert res["calls"] == expect, (r, res["calls"])
