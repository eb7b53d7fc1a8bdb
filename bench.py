"""Benchmark: RWKV-7 2.9B grouped-U8 (SG8 g128) greedy decode tok/s on B200.

One JSON line on rank 0.  A *step* is one decode token at batch 1 (the whole
packed RWKV-7 token step: embedding, 32 layers of time mix + channel mix,
head, greedy argmax).  Inputs are resident in HBM before timing; the weights
streamed per token (~3 GB) are far larger than the 126 MB L2, so no flush is
needed between steps.

Multi-GPU (torchrun): decode does not shard at batch 1 — every rank runs an
independent replica (its own model copy and session), ``scaling: "weak"``;
``value`` = tokens decoded by all ranks / max-over-ranks device time.

``e2e`` is the same metric through the drop-in plugin
(``create_backend("cuda_b200").decode_greedy`` with a token callback): every
token's argmax is read back to the host and the token is sent to the device
through the C ABI before the next step.  The timed regions sit inside NVTX
ranges ``timed`` and ``e2e``.

``batched`` (key of the same line) is the bs64 leg: ``--sessions`` sessions
decoded together through ``B200BatchEngine`` (tcgen05 batched GEMMs), one
step = one token for every session.

``prefill`` is the sequence-prefill leg (``--prefill-sessions`` sessions x
``--prefill-tokens`` tokens through ``B200BatchEngine.prefill``).

``tp`` is the 7.2B leg (``--tp-sessions`` sessions, tensor-parallel over the
ranks; unsplit at one GPU), with, at one GPU, the 7.2B sequence prefill of
``--tp-prefill-tokens`` tokens per session (``tp.prefill``, reported against
HBM and against tensor throughput).  ``lut2`` holds the LUT2 (``TR2\x04``)
legs of the same 2.9B shape, ``small`` the 0.1B-shaped bs1 leg (a
``--small-prompt``-token prompt, then ``--small-steps`` greedy tokens).

``--impl reference`` times the reference's own C kernels (built from its
sources into ``oracle/_ref``) driving the packed RWKV-7 forward on the host
cores, on the same workload and metric (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "ssd-rwkv-engine_b200"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from rwkv_b200 import replicas  # noqa: E402

SEED = 2026
PROMPT = 8


def _env_int(k: str, d: int) -> int:
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def _nvtx_push(name: str) -> None:
    """Named range around a timed region, so a profiler can select its launches."""
    try:
        torch.cuda.nvtx.range_push(name)
    except Exception:
        pass


def _nvtx_pop() -> None:
    try:
        torch.cuda.nvtx.range_pop()
    except Exception:
        pass


def _peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def _tflops_peak() -> tuple[float, str]:
    """Sustained dense bf16 tensor throughput (the denominator of a flop roofline for a long step)."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured sustained bf16"
        except Exception:
            pass
    return 1400.0, "fallback sustained bf16"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", ",".join(map(str, self.gpus))],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sms)) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


def metric_name(args, bs: int = 1) -> str:
    """The headline metric string, identical in both arms."""
    codec = "U8" if args.policy == "sg8" else "LUT2"
    return f"RWKV-7 {args.config} {codec} decode tok/s (bs{bs})"


def cpu_threads() -> int:
    """Set the CPU library's OpenMP threads to all physical host cores
    explicitly (torchrun exports OMP_NUM_THREADS=1 to every rank) and return
    the count in effect."""
    from oracle import kernels as ok

    impl = "reference" if ok.ref_available() else "oracle"
    return ok.set_threads(ok.host_threads(), impl)


CPU_SAMPLE = ("the oracle's restatement of forward_block_packed (NumPy fp32 glue; the reference's Python "
              "package cannot travel to the GPU host) calling the reference's own lut2_gather.c kernels "
              "(oracle/_ref, built -O3 -mavx2 -mfma -fopenmp from its source) for every GEMV")


def bytes_per_token(pack, shape) -> int:
    """Algorithmic HBM bytes of one decode token: every packed matrix read once
    (embedding: one row; layer 0's unused v1/v2 excluded), skeleton vectors,
    and the recurrent state read + written."""
    C, L, H = shape.n_embd, shape.n_layer, shape.n_head
    tot = 0
    for n, e in pack.items():
        if n in ("blocks.0.att.v1", "blocks.0.att.v2", "blocks.0.att.v0"):
            continue
        p = e.payload
        nb = int(p.numel() * p.element_size()) if isinstance(p, torch.Tensor) else (
            len(p) if isinstance(p, (bytes, bytearray)) else int(np.asarray(p).nbytes))
        if n == "emb.weight":
            g = 128
            nb = C + (C // g) * 8
        tot += nb
    state = L * (2 * C + H * 64 * 64) * 4
    return tot + 2 * state


def run_reference(args, shape, rank: int) -> dict:
    """The reference's C kernels (oracle/_ref) driving the packed forward on
    all physical host cores: the same seeded model and prompt as the b200 arm,
    then greedy decode steps, each step one token (bounded by a time budget)."""
    from oracle import kernels as ok
    from oracle.forward import OracleRWKV7
    from rwkv_b200 import synth

    if not ok.ref_available():
        return {"impl": "reference", "unavailable": "reference C kernels (oracle/_ref) not built"}
    cores = cpu_threads()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    pack = synth.pack_to_host(synth.make_pack_streaming(shape, SEED, dev, policy=args.policy))
    if dev == "cuda":
        torch.cuda.empty_cache()
    model = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size,
                        impl="reference")
    state = model.zero_state()
    prompt = synth.seeded_prompt(PROMPT, shape.vocab, SEED)
    for t in prompt:
        logits = model.forward_token(t, state)
    tok = int(np.argmax(logits))
    for _ in range(args.warmup):
        logits = model.forward_token(tok, state)
        tok = int(np.argmax(logits))
    t0 = time.perf_counter()
    n = 0
    for _ in range(args.steps):
        logits = model.forward_token(tok, state)
        tok = int(np.argmax(logits))
        n += 1
        if time.perf_counter() - t0 > args.ref_budget_s:
            break
    dt = time.perf_counter() - t0
    v = n / dt
    return {"metric": metric_name(args), "value": v,
            "unit": "tok/s", "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 * dt / n,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"rwkv7-{args.config} {args.policy} bs1 greedy decode, {PROMPT}-token prompt",
                       "batch": 1},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{n} decode tokens (time budget {args.ref_budget_s}s) after "
                                       f"{args.warmup} warm-up tokens, {cores} OpenMP threads: " + CPU_SAMPLE},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_batched(eng, args, shape, bpt: int, dev, stream, world: int, rank: int) -> dict:
    """The batched leg: ``args.sessions`` sessions decoded together (tcgen05 GEMMs
    for SG8 packs, CUDA-core products for TR2\x04 packs).

    One step = one token for every session.  Algorithmic bytes per step: the
    weights once (the batch-1 token bytes less its state traffic), plus the
    recurrent state read and written for every session and one embedding row
    per session."""
    import torch.distributed as dist

    nb = eng.batch
    C, L, H = shape.n_embd, shape.n_layer, shape.n_head
    state = L * (2 * C + H * 64 * 64) * 4
    emb_row = C + (C // 128) * 8
    step_bytes = bpt - 2 * state + nb * 2 * state + (nb - 1) * emb_row
    # global sessions [rank * nb, (rank + 1) * nb): a session's prompt does not depend on the world size
    prompts = [synth_prompt(PROMPT, shape.vocab, replicas.session_seed(SEED, g))
               for g in replicas.session_range(nb, rank, world)]
    for pos in range(PROMPT):
        eng.forward([p[pos] for p in prompts])
    out = torch.empty((max(args.batch_steps, args.warmup) + 1) * nb, dtype=torch.int32, device=dev)
    eng.decode_greedy_async(args.warmup, out)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("timed_batched")
    t0.record(stream)
    eng.decode_greedy_async(args.batch_steps, out)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    ms = replicas.max_over_ranks(t0.elapsed_time(t1))
    ms_step = ms / args.batch_steps
    # end to end: per step the session tokens go host->device through the C ABI
    # and the argmax ids come back device->host
    e_steps = min(16, args.batch_steps)
    toks = eng.logits.argmax(dim=1).to(torch.int32).cpu().tolist()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        eng.forward(toks)
        toks = eng.logits.argmax(dim=1).to(torch.int32).cpu().tolist()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e_ms = replicas.max_over_ranks(e0.elapsed_time(e1))
    peak, peak_kind = _peaks()
    achieved = step_bytes / (ms_step / 1e3) / 1e9
    eng.close()
    codec = "U8" if args.policy == "sg8" else "LUT2"
    return {"metric": f"RWKV-7 {args.config} {codec} decode tok/s (bs{nb})", "value": nb * world / (ms_step / 1e3),
            "unit": "tok/s", "sessions_per_gpu": nb, "steps": args.batch_steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "gpu_launches": eng.launches_per_step * args.batch_steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes_per_step": step_bytes,
                         "what": f"whole batched step ({eng.launches_per_step} launches in one CUDA graph): "
                                 f"weights once + {nb} sessions' state read and written; peak: {peak_kind} "
                                 "HBM copy bandwidth"},
            "e2e": {"value": e_steps * nb * world / (e_ms / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * nb, "d2h_bytes_per_step": 4 * nb, "steps": e_steps,
                    "how": "B200BatchEngine.forward(host ids) + per-session argmax read back each step"}}


def run_prefill(eng, args, shape, bpt: int, dev, stream, world: int, rank: int) -> dict:
    """Sequence prefill leg: ``args.prefill_sessions`` sessions consume
    ``args.prefill_tokens`` seeded tokens each (``B200BatchEngine.prefill``:
    chunks of 64 / sessions positions per GEMM), timed from the host call
    (tokens copied to the device per chunk) to the last position's logits."""
    nb, n = eng.batch, args.prefill_tokens
    prompts = [synth_prompt(n, shape.vocab, replicas.session_seed(SEED + 1, g))
               for g in replicas.session_range(nb, rank, world)]
    warm = [p[:64] for p in prompts]
    eng.prefill(warm)  # builds the chunk plan and graph
    eng.reset()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("timed_prefill")
    t0.record(stream)
    eng.prefill(prompts)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    ms = replicas.max_over_ranks(t0.elapsed_time(t1))
    chunk = max(1, 64 // nb)
    chunks = n // chunk if chunk > 1 else 0
    C, L, H = shape.n_embd, shape.n_layer, shape.n_head
    state = L * (2 * C + H * 64 * 64) * 4
    emb_row = C + (C // 128) * 8
    head = shape.vocab * C + shape.vocab * (C // 128) * 8
    weights = bpt - 2 * state - emb_row - head  # projections and adapters, once per chunk
    alg = chunks * (weights + nb * 2 * state + nb * chunk * emb_row) + head
    peak, peak_kind = _peaks()
    achieved = alg / (ms * 1e-3) / 1e9
    eng.close()
    return {"metric": f"RWKV-7 {args.config} U8 prefill tok/s ({nb} sessions x {n} tokens)",
            "value": nb * n * world / (ms * 1e-3), "unit": "tok/s", "ms": ms, "sessions_per_gpu": nb,
            "tokens_per_session": n, "chunk_positions": chunk,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes": alg,
                         "what": f"weights once per chunk of {chunk} positions x {nb} sessions (tcgen05 GEMM rows), "
                                 f"state read and written per chunk and session, head once; peak: {peak_kind}"},
            "e2e": {"value": nb * n * world / (ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 4 * nb * chunk,
                    "d2h_bytes_per_step": 0, "how": "B200BatchEngine.prefill(host prompts): tokens copied per chunk"}}


def run_lut2(args, shape, dev, stream, world: int, rank: int) -> dict:
    """The LUT2 legs (the 2.9B LUT2 configuration: 2-bit codes into a 4-entry
    fp16 codebook per 64-column group): the same seeded model encoded as
    ``TR2\x04``, greedy decode at batch 1 (``args.lut2_steps`` tokens, one
    launch) and the batched step at ``args.lut2_sessions`` sessions."""
    import argparse

    import torch.distributed as dist
    from rwkv_b200 import synth
    from rwkv_b200.engine import B200BatchEngine, B200Engine, ModelUpload

    largs = argparse.Namespace(**vars(args))
    largs.policy = "lut2"
    pack = synth.make_pack_streaming(shape, SEED + rank, dev, policy="lut2")
    bpt = bytes_per_token(pack, shape)
    model = ModelUpload(pack, dev)
    del pack
    torch.cuda.empty_cache()
    eng = B200Engine(model, device=dev.index)
    out = {}
    try:
        prompt = synth.seeded_prompt(PROMPT, shape.vocab, SEED + rank)
        eng.forward(prompt)
        first = int(torch.argmax(eng.logits).item())
        ids = torch.empty(max(args.lut2_steps, args.warmup) + 8, dtype=torch.int32, device=dev)
        eng.decode_greedy_async(first, args.warmup, ids)
        torch.cuda.synchronize(dev)
        nxt = int(ids[args.warmup - 1].item())
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        eng.decode_greedy_async(nxt, args.lut2_steps, ids)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        ms = replicas.max_over_ranks(t0.elapsed_time(t1))
        ms_step = ms / args.lut2_steps
        peak, peak_kind = _peaks()
        achieved = bpt / (ms_step / 1e3) / 1e9
        out["bs1"] = {"metric": metric_name(largs), "value": args.lut2_steps * world / (ms / 1e3), "unit": "tok/s",
                      "steps": args.lut2_steps, "ms_per_step": ms_step,
                      "path": "persistent kernel" if eng.persistent_active else "multi-kernel CUDA graph",
                      "gpu_launches": (eng.launches_per_step * args.lut2_steps) if eng.launches_per_step else 1,
                      "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                   "frac": achieved / peak, "traffic": None, "algorithmic_bytes_per_step": bpt,
                                   "what": f"bs1 decode: algorithmic bytes/token {bpt} (TR2x04 projections and head, "
                                           f"SG8 adapters and embedding row, state) / device time per token; peak: "
                                           f"{peak_kind} HBM copy bandwidth"}}
    finally:
        eng.close()
    if args.lut2_sessions > 0:
        beng = B200BatchEngine(model, args.lut2_sessions, device=dev.index)
        out["batched"] = run_batched(beng, largs, shape, bpt, dev, stream, world, rank)
    del model
    torch.cuda.empty_cache()
    return out


def run_tp(args, dev, stream, world: int, rank: int) -> dict:
    """Tensor-parallel leg: ``args.tp_sessions`` sessions of the ``args.tp_config``
    model decoded with the model split over all ranks (heads, FFN rows and
    vocabulary rows; two NCCL all-reduces per layer and one all-gather of the
    argmax bests per step, captured with the step in one CUDA graph).  At one
    GPU the same sessions run on the unsplit batched engine.  Total work is
    fixed as the rank count grows (strong scaling).  Algorithmic bytes per step:
    the weights once over all ranks plus every session's state read and
    written; the peak is the ranks' summed HBM bandwidth."""
    from rwkv_b200 import synth, tp
    from rwkv_b200.engine import B200BatchEngine

    shape = synth.PRESETS[args.tp_config]
    nb = args.tp_sessions
    if world > 1:
        plan = tp.plan(shape, rank, world)
        local = synth.make_pack_streaming(shape, SEED + 7, dev, policy="sg8",
                                          transform=lambda n, e: tp.shard_entry(n, e, plan))
        eng = tp.B200TPBatchEngine(local, nb, device=dev, shard_plan=plan, use_graph=True,
                                   exchange=args.tp_exchange)
    else:
        local = synth.make_pack_streaming(shape, SEED + 7, dev, policy="sg8")
        eng = B200BatchEngine(local, nb, device=dev)
    bpt_local = bytes_per_token(local, shape) if world == 1 else None
    del local
    torch.cuda.empty_cache()
    prompts = [synth_prompt(16, shape.vocab, replicas.session_seed(SEED + 7, g)) for g in range(nb)]
    for pos in range(16):
        eng.forward([p[pos] for p in prompts])
    out = torch.empty((max(args.tp_steps, args.warmup) + 1) * nb, dtype=torch.int32, device=dev)
    eng.decode_greedy_async(args.warmup, out)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("timed_tp")
    t0.record(stream)
    eng.decode_greedy_async(args.tp_steps, out)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    ms = replicas.max_over_ranks(t0.elapsed_time(t1))
    ms_step = ms / args.tp_steps
    # end to end: greedy ids of every step copied back to the host
    e_steps = min(8, args.tp_steps)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ids = eng.decode_greedy(e_steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e_ms = replicas.max_over_ranks(e0.elapsed_time(e1))
    C, L, H = shape.n_embd, shape.n_layer, shape.n_head
    state = L * (2 * C + H * 64 * 64) * 4
    emb_row = C + (C // 128) * 8
    weights = shape.weights_per_token() * 1.0625  # SG8 g128, embedding row excluded
    step_bytes = int(weights + nb * (2 * state + emb_row))
    peak, peak_kind = _peaks()
    achieved = step_bytes / (ms_step / 1e3) / 1e9
    launches = eng.launches_per_step
    prefill = None
    if world == 1 and args.tp_prefill_tokens > 0:
        prefill = run_tp_prefill(eng, args, shape, nb, dev, stream)
    eng.close()
    return {"metric": f"RWKV-7 {args.tp_config} U8 decode tok/s (bs{nb}, tensor-parallel x{world})",
            "value": nb / (ms_step / 1e3), "unit": "tok/s", "n_gpus": world, "sessions": nb, "scaling": "strong",
            "steps": args.tp_steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "gpu_launches": launches * args.tp_steps,
            "collectives_per_step": (2 * L + 1) if world > 1 else 0,
            "exchange": args.tp_exchange if world > 1 else None,
            "allreduce_bytes": nb * C * 4 if world > 1 else 0,
            "parallelism": f"tp{world}" if world > 1 else "single GPU (unsplit)",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
                         "frac": achieved / (peak * world), "traffic": None, "algorithmic_bytes_per_step": step_bytes,
                         "what": f"weights once over all ranks + {nb} sessions' state read and written per step; "
                                 f"peak: {world} x {peak_kind} HBM copy bandwidth"},
            "e2e": {"value": e_steps * nb / (e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 4 * nb, "steps": e_steps,
                    "how": "decode_greedy: ids of every step copied to the host"},
            "ids_checksum": int(ids.astype("int64").sum()), "bytes_per_token_unsplit": bpt_local,
            "prefill": prefill if world == 1 else {"skipped": "sequence prefill runs on the unsplit engine (N = 1)"}}


def run_tp_prefill(eng, args, shape, nb: int, dev, stream) -> dict:
    """Sequence prefill of the TP leg's model at one GPU: ``nb`` sessions x
    ``args.tp_prefill_tokens`` seeded tokens through ``B200BatchEngine.prefill``
    from a fresh state.  Reported against HBM (weights once per chunk) and
    against tensor throughput (the model's matmul flops, two per weight and
    token, over the measured sustained bf16 peak)."""
    n = args.tp_prefill_tokens
    prompts = [synth_prompt(n, shape.vocab, replicas.session_seed(SEED + 11, g)) for g in range(nb)]
    eng.reset()
    eng.prefill([p[:64] for p in prompts])  # builds the chunk plan and graph
    eng.reset()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("timed_tp_prefill")
    t0.record(stream)
    eng.prefill(prompts)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    ms = t0.elapsed_time(t1)
    tokens = nb * n
    chunk = max(1, 64 // nb)
    C, L, H = shape.n_embd, shape.n_layer, shape.n_head
    state = L * (2 * C + H * 64 * 64) * 4
    emb_row = C + (C // 128) * 8
    head = shape.vocab * C + shape.vocab * (C // 128) * 8
    weights = shape.weights_per_token() * 1.0625 - head  # projections and adapters, once per chunk
    alg = (n // chunk) * (weights + nb * 2 * state + nb * chunk * emb_row) + head
    peak, peak_kind = _peaks()
    flops = 2.0 * (shape.weights_per_token() - shape.vocab * C) * tokens + 2.0 * shape.vocab * C * nb
    tpk, tpk_kind = _tflops_peak()
    return {"metric": f"RWKV-7 {args.tp_config} U8 prefill tok/s ({nb} sessions x {n} tokens)",
            "value": tokens / (ms * 1e-3), "unit": "tok/s", "ms": ms, "sessions": nb, "tokens_per_session": n,
            "chunk_positions": chunk,
            "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None, "algorithmic_bytes": alg,
                         "what": f"weights once per chunk of {chunk} positions x {nb} sessions, state per chunk and "
                                 f"session, head once; peak: {peak_kind} HBM copy bandwidth"},
            "roofline_flops": {"bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": tpk,
                               "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / tpk,
                               "algorithmic_flops": flops,
                               "what": f"2 flops per projection weight per token (the head once per session); "
                                       f"peak: {tpk_kind} (the GEMMs run as integer MMAs on 3 digit rows per input)"}}


def run_small(args, dev, stream, world: int, rank: int) -> dict:
    """The 0.1B-shaped configuration: a seeded ``args.small_prompt``-token
    prompt, then ``args.small_steps`` greedy tokens at batch 1 on the
    persistent kernel (each rank an independent replica)."""
    from rwkv_b200 import synth
    from rwkv_b200.engine import B200Engine, ModelUpload

    shape = synth.PRESETS["0.1b"]
    pack = synth.make_pack_streaming(shape, SEED + 13 + rank, dev, policy="sg8")
    bpt = bytes_per_token(pack, shape)
    model = ModelUpload(pack, dev)
    del pack
    eng = B200Engine(model, device=dev.index)
    try:
        prompt = synth_prompt(args.small_prompt, shape.vocab, SEED + 13 + rank)
        eng.forward(prompt[:8])  # first launch of each path outside the timed regions
        eng.reset()
        torch.cuda.synchronize(dev)
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        eng.forward(prompt)
        p1.record(stream)
        torch.cuda.synchronize(dev)
        pf_ms = replicas.max_over_ranks(p0.elapsed_time(p1))
        first = int(torch.argmax(eng.logits).item())
        ids = torch.empty(args.small_steps + 8, dtype=torch.int32, device=dev)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        eng.decode_greedy_async(first, args.small_steps, ids)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        ms = replicas.max_over_ranks(t0.elapsed_time(t1))
        persistent = eng.persistent_active
    finally:
        eng.close()
    ms_step = ms / args.small_steps
    peak, peak_kind = _peaks()
    achieved = bpt / (ms_step / 1e3) / 1e9
    return {"metric": "RWKV-7 0.1b U8 decode tok/s (bs1)", "value": args.small_steps * world / (ms / 1e3),
            "unit": "tok/s", "steps": args.small_steps, "ms_per_step": ms_step,
            "prompt_tokens": args.small_prompt, "prompt_tok_s": args.small_prompt * world / (pf_ms / 1e3),
            "path": "persistent kernel" if persistent else "multi-kernel CUDA graph",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes_per_step": bpt,
                         "what": f"bs1 decode: algorithmic bytes/token {bpt} / device time per token; peak: "
                                 f"{peak_kind} HBM copy bandwidth"}}


def synth_prompt(n: int, vocab: int, seed: int) -> list[int]:
    from rwkv_b200 import synth

    return synth.seeded_prompt(n, vocab, seed)


def cpu_baseline(pack_dev, shape, args, gpu_ids: list[int]) -> dict:
    """The same model on the host cores (reference C kernels inside the
    oracle's forward), from the same prompt: greedy ids compared with the GPU
    decode's ids (``ids_match_oracle``) and decode tokens per second."""
    from oracle import kernels as ok
    from oracle.forward import OracleRWKV7
    from rwkv_b200 import synth

    impl = "reference" if ok.ref_available() else "oracle"
    cores = cpu_threads()
    pack = synth.pack_to_host(pack_dev)
    model = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size, impl=impl)
    st = model.zero_state()
    for t in synth.seeded_prompt(PROMPT, shape.vocab, SEED):
        logits = model.forward_token(t, st)
    tok = int(np.argmax(logits))
    ids = [tok]
    t0 = time.perf_counter()
    n = 0
    while n < 64:
        logits = model.forward_token(tok, st)
        tok = int(np.argmax(logits))
        ids.append(tok)
        n += 1
        if time.perf_counter() - t0 > args.cpu_budget_s:
            break
    dt = time.perf_counter() - t0
    k = min(len(ids), len(gpu_ids))
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} decode tokens of the same {args.config} {args.policy} model after the same "
                      f"{PROMPT}-token prompt ({dt:.1f}s), {cores} OpenMP threads: "
                      + (CPU_SAMPLE if impl == "reference" else "the oracle's C GEMVs"),
            "ids_compared": k, "ids_match": ids[:k] == [int(v) for v in gpu_ids[:k]]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="2.9b", choices=["tiny", "0.1b", "2.9b", "7.2b", "2.9b-l4"])
    ap.add_argument("--policy", default="sg8", choices=["sg8", "lut2"])
    ap.add_argument("--e2e-steps", type=int, default=256)
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--ref-budget-s", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sessions", type=int, default=64, help="batched-decode sessions (0: skip the batched leg)")
    ap.add_argument("--batch-steps", type=int, default=64)
    ap.add_argument("--prefill-tokens", type=int, default=512, help="prefill leg: tokens per session (0: skip)")
    ap.add_argument("--prefill-sessions", type=int, default=8)
    ap.add_argument("--tp-prefill-tokens", type=int, default=4096,
                    help="tp leg at one GPU: sequence prefill tokens per session (0: skip)")
    ap.add_argument("--small-steps", type=int, default=256, help="0.1B leg: greedy tokens after the prompt (0: skip)")
    ap.add_argument("--small-prompt", type=int, default=512, help="0.1B leg: prompt tokens")
    ap.add_argument("--lut2-steps", type=int, default=64, help="LUT2 leg: bs1 decode tokens (0: skip the leg)")
    ap.add_argument("--lut2-sessions", type=int, default=64, help="LUT2 leg: batched sessions (0: bs1 only)")
    ap.add_argument("--tp-config", default="7.2b", choices=["tiny", "7.2b", "7.2b-l4", "2.9b"],
                    help="tensor-parallel leg: model split over all ranks")
    ap.add_argument("--tp-sessions", type=int, default=8, help="tensor-parallel leg sessions (0: skip the leg)")
    ap.add_argument("--tp-steps", type=int, default=32)
    ap.add_argument("--tp-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel exchange: the engine's peer-memory kernels or NCCL through the host callback")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local = _env_int("LOCAL_RANK", 0)
    from rwkv_b200 import synth

    shape = synth.PRESETS[args.config]

    if args.impl == "reference":
        if rank == 0:
            if torch.cuda.is_available():
                torch.cuda.set_device(local)
            print(json.dumps(run_reference(args, shape, rank)), flush=True)
        return

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from rwkv_b200.backend import PackProvider, create_backend

    pack = synth.make_pack_streaming(shape, SEED + rank, dev, policy=args.policy)
    bpt = bytes_per_token(pack, shape)
    # the engine under test is the one the drop-in plugin builds from a provider
    backend = create_backend("cuda_b200")
    backend.load_pack(None, f"cuda:{local}")
    provider = PackProvider(pack)
    backend.prepare_provider(provider)
    eng = backend._engine
    cpu_pack = pack if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    batch_eng = prefill_eng = None
    if args.sessions > 0 or (args.policy == "sg8" and args.prefill_tokens > 0):
        from rwkv_b200.engine import B200BatchEngine

        if args.sessions > 0:
            batch_eng = B200BatchEngine(backend._model, args.sessions, device=local)
        if args.policy == "sg8" and args.prefill_tokens > 0:
            prefill_eng = B200BatchEngine(backend._model, args.prefill_sessions, device=local)
    del pack
    provider.pack, provider._fused = {}, {}
    torch.cuda.empty_cache()

    stream = torch.cuda.current_stream(dev)
    prompt = synth.seeded_prompt(PROMPT, shape.vocab, SEED + rank)
    eng.forward(prompt)
    first = int(torch.argmax(eng.logits).item())
    out = torch.empty(max(args.steps, args.warmup) + 8, dtype=torch.int32, device=dev)
    eng.decode_greedy_async(first, args.warmup, out)
    torch.cuda.synchronize(dev)
    nxt = int(out[args.warmup - 1].item())
    # the greedy sequence after the prompt: first, the warm-up ids, then the timed ids
    gpu_ids = [first] + [int(v) for v in out[:args.warmup].cpu().tolist()]

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(list(range(world)) if rank == 0 else [])
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("timed")
    t0.record(stream)
    eng.decode_greedy_async(nxt, args.steps, out)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    ms = t0.elapsed_time(t1)
    gpu_ids += [int(v) for v in out[:args.steps].cpu().tolist()]
    clk = clocks.stop() if rank == 0 else {}
    ms = replicas.max_over_ranks(ms)
    if world > 1:
        dist.barrier()
    total_tokens = args.steps * world
    value = total_tokens / (ms / 1e3)
    ms_step = ms / args.steps

    # end to end through the plugin: CudaB200Backend.decode_greedy with a
    # per-token callback; every step's id crosses to the host (mapped pinned
    # memory) and the callback sees it before the call returns
    e2e_steps = min(args.e2e_steps, args.steps)
    state = backend.prefill_tokens(prompt)
    emitted: list[int] = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    _nvtx_push("e2e")
    e0.record(stream)
    backend.decode_greedy(state, provider, e2e_steps, None, token_callback=emitted.append)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    _nvtx_pop()
    assert len(emitted) == e2e_steps
    e2e_ms = replicas.max_over_ranks(e0.elapsed_time(e1))
    e2e_val = e2e_steps * world / (e2e_ms / 1e3)

    batched = run_batched(batch_eng, args, shape, bpt, dev, stream, world, rank) if batch_eng is not None else None
    prefill = run_prefill(prefill_eng, args, shape, bpt, dev, stream, world, rank) if prefill_eng is not None else None
    lut2 = None
    if args.lut2_steps > 0 and args.policy == "sg8" and args.config in ("2.9b", "2.9b-l4", "0.1b", "tiny"):
        # the LUT2 configuration of the same shape; a failure is reported in the line
        try:
            lut2 = run_lut2(args, shape, dev, stream, world, rank)
        except Exception as exc:  # noqa: BLE001
            lut2 = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.synchronize(dev)
    small = None
    if args.small_steps > 0 and args.policy == "sg8":
        try:
            small = run_small(args, dev, stream, world, rank)
        except Exception as exc:  # noqa: BLE001
            small = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.synchronize(dev)
    tpres = None
    if args.tp_sessions > 0:
        # the tensor-parallel leg must not take the line's other results with it:
        # a failure there is reported in the line instead
        try:
            tpres = run_tp(args, dev, stream, world, rank)
        except Exception as exc:  # noqa: BLE001
            tpres = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.synchronize(dev)

    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = bpt / (ms_step / 1e3) / 1e9
        # DRAM bytes of the launch from the committed ncu capture (per token x
        # tokens of this launch), null when no capture exists for this workload
        traffic = None
        tf = REPO / "profiles" / f"decode_{args.config}_{args.policy}_traffic.json"
        if tf.is_file():
            try:
                traffic = int(json.loads(tf.read_text())["dram_bytes_per_step"]) * args.steps
            except Exception:
                traffic = None
        res = {
            "metric": metric_name(args),
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (u8/2-bit weights)", "data": "synthetic (seeded random RWKV-7 weights, reference codecs)",
            "config": {"workload": f"rwkv7-{args.config} {args.policy} bs1 greedy decode, {PROMPT}-token prompt",
                       "model": f"rwkv7-{args.config}", "global_batch": world, "batch_per_gpu": 1,
                       "n_layer": shape.n_layer, "d_model": shape.n_embd, "ffn": shape.ffn, "vocab": shape.vocab,
                       "codec": "SG8 g128" if args.policy == "sg8" else "TR2x04 g64 (+SG8 g128 adapters/emb)",
                       "parallelism": f"replicas x{world}",
                       "l2": "weights per token (%.2f GB) >> 126 MB L2; no flush needed" % (bpt / 1e9)},
            "gpu_launches": (eng.launches_per_step * args.steps + 1) if eng.launches_per_step
            else (args.steps + 65535) // 65536,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "algorithmic_bytes": bpt * args.steps,
                         "what": f"decode_kernel, one persistent launch decoding {args.steps} tokens: "
                                 f"algorithmic bytes/token {bpt} x tokens / CUDA-event duration of the launch; "
                                 f"peak: {peak_kind} HBM copy bandwidth"},
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8,
                    "steps": e2e_steps,
                    "how": "cuda_b200 plugin decode_greedy with a token callback: one persistent launch for the "
                           "whole generation; per token the device writes the id and a count (8 B) into mapped "
                           "pinned host memory and reads the host's cancel word (4 B); the callback runs on the "
                           "host as each id arrives"},
            "clocks": clk,
        }
        if batched is not None:
            res["batched"] = batched
        if prefill is not None:
            res["prefill"] = prefill
        if tpres is not None:
            res["tp"] = tpres
        if lut2 is not None:
            res["lut2"] = lut2
        if small is not None:
            res["small"] = small
        if cpu_pack is not None:
            backend.close()
            cb = cpu_baseline(cpu_pack, shape, args, gpu_ids)
            res["ids_match_oracle"] = cb.pop("ids_match")
            res["ids_compared"] = cb.pop("ids_compared")
            res["cpu_baseline"] = cb
        print(json.dumps(res), flush=True)
    backend.close()
    if world > 1:
        try:
            dist.barrier()
        finally:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
