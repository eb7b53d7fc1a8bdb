"""Multi-GPU decode by replicas: one process per GPU, each holding its own copy
of the model and decoding its own sessions, with no collective on the data
path (the reference runs independent sessions per device; tensor splitting,
``rwkv_b200.tp``, is for models whose step should be spread over several GPUs,
such as the 7.2B one).

The host logic here is what every rank runs around the device work:

* ``session_range`` — the contiguous block of global session ids a rank serves
  (weak scaling: sessions per rank fixed, ids stable across world sizes);
* ``session_seed`` — the seed of a global session, so a session decodes the
  same tokens whichever rank serves it;
* ``max_over_ranks`` — the job's time is the slowest rank's (all-reduce MAX);
* ``gather_ranks`` — per-rank results collected in rank order (for checking
  that every session decoded);
* ``missing_peers`` — a heartbeat through the rendezvous store: before a step's
  collectives every rank posts its key and waits a short time for the others,
  so a rank that left between steps is seen on the host (and the step is not
  started) instead of a collective waiting on it.

Every collective goes through ``torch.distributed`` with the process group the
caller initialised (``nccl`` on the GPUs, ``gloo`` in the CPU tests); every
rank calls the same collectives in the same order.
"""

from __future__ import annotations

import datetime

import torch
import torch.distributed as dist


def world() -> tuple[int, int]:
    """(rank, world size); (0, 1) without an initialised process group."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def session_range(sessions_per_rank: int, rank: int, world_size: int) -> range:
    """Global session ids served by ``rank``: ``[rank * n, (rank + 1) * n)``."""
    if sessions_per_rank < 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad session split: n={sessions_per_rank} rank={rank} world={world_size}")
    return range(rank * sessions_per_rank, (rank + 1) * sessions_per_rank)


def session_seed(base_seed: int, session: int) -> int:
    """Seed of global session ``session`` (independent of the rank serving it)."""
    return (int(base_seed) + 7919 * int(session)) % (2**31 - 1)


def _device_for_backend() -> torch.device:
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(value: float) -> float:
    """The maximum of ``value`` over all ranks (every rank gets it)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_device_for_backend())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_ranks(values: list[int]) -> list[list[int]]:
    """All ranks' integer lists, in rank order (every rank gets all of them).
    Lists may differ in length."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [list(values)]
    dev = _device_for_backend()
    ws = dist.get_world_size()
    n = torch.tensor([len(values)], dtype=torch.int64, device=dev)
    lens = [torch.zeros_like(n) for _ in range(ws)]
    dist.all_gather(lens, n)
    cap = int(max(int(x.item()) for x in lens))
    buf = torch.zeros(cap, dtype=torch.int64, device=dev)
    if values:
        buf[: len(values)] = torch.tensor(values, dtype=torch.int64, device=dev)
    parts = [torch.zeros_like(buf) for _ in range(ws)]
    dist.all_gather(parts, buf)
    return [p[: int(l.item())].tolist() for p, l in zip(parts, lens)]


def missing_peers(store, step: int, rank: int, world_size: int, timeout_s: float = 2.0) -> list[int]:
    """Post this rank's heartbeat for ``step`` and return the ranks whose
    heartbeat did not arrive within ``timeout_s`` (empty: all present)."""
    store.set(f"rwkvb/alive/{int(step)}/{int(rank)}", "1")
    missing = []
    for r in range(world_size):
        if r == rank:
            continue
        try:
            store.wait([f"rwkvb/alive/{int(step)}/{r}"], datetime.timedelta(seconds=timeout_s))
        except Exception:
            missing.append(r)
    return missing
