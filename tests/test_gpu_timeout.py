"""A bounded device wait that runs out: the tensor-parallel peer exchange of a
rank whose peer never arrives.

One process, one GPU, no second rank: rank 0 of a two-rank peer-exchange
engine gets its own exchange buffer and, as rank 1's buffer, a zeroed device
buffer whose flags nothing ever sets.  The exchange kernel's wait gives up
after its wall-time limit (100 ms here, engine flag bits 16..19), the step's
later exchanges return at once, and the next synchronising call reports
``RWKVB_ETIMEOUT`` and clears the engine's error word.  The context stays
usable: a second call times out again the same way (nothing sticky) and an
ordinary engine decodes afterwards.  No kernel waits on another launch; the
flag that would release the wait is simply never written.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)

from rwkv_b200 import native, synth, tp  # noqa: E402
from rwkv_b200.engine import B200BatchEngine, ModelUpload  # noqa: E402
from rwkv_b200.native import RwkvbError  # noqa: E402

LIMIT_100MS = 1  # flag bits 16..19: exchange wait limit in units of 100 ms


def test_peer_exchange_wait_gives_up_with_etimeout():
    lib = native.lib()
    dev = torch.device("cuda", 0)
    shape = synth.PRESETS["tiny"]
    pack = synth.make_pack(synth.generate_state_dict(shape, 11, "cpu"), policy="sg8")
    local, plan = tp.shard_pack(pack, 0, 2)
    nb = 2
    with torch.cuda.device(dev):
        model = ModelUpload(local, dev)
        nbytes = ctypes.c_uint64()
        native.check(lib.rwkvb_batch_tp_exchange_bytes(ctypes.byref(model.md), nb, ctypes.byref(nbytes)),
                     "rwkvb_batch_tp_exchange_bytes")
        own = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=dev)
        absent = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=dev)  # rank 1: never arrives
        peers = (ctypes.c_void_p * 2)(own.data_ptr(), absent.data_ptr())

        def unused(kind, send, recv, nbytes_, stream, user):  # the peer exchange replaces the callback
            raise AssertionError("collective callback called under the peer exchange")

        cfn = native.COLLECTIVE_FN(unused)
        desc = native.TPDesc(0, 2, plan.v0, cfn, None, None)
        desc.peer = peers
        h = ctypes.c_void_p()
        flags = native.FLAG_NO_GRAPH | (LIMIT_100MS << 16)
        native.check(lib.rwkvb_batch_create_tp(ctypes.byref(model.md), nb, ctypes.byref(desc), flags,
                                               ctypes.byref(h)), "rwkvb_batch_create_tp")
        try:
            s = torch.cuda.current_stream(dev).cuda_stream
            out = np.zeros((1, nb), dtype=np.int32)
            optr = out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
            toks = (ctypes.c_int32 * nb)(3, 5)
            assert lib.rwkvb_batch_forward(h, toks, s) == native.RWKVB_OK  # asynchronous: no status yet
            st = lib.rwkvb_batch_decode_greedy(h, 1, optr, s)  # synchronises and reads the error word
            assert st == native.RWKVB_ETIMEOUT, lib.rwkvb_status_string(st).decode()
            # the error word was cleared: the next step waits (and gives up) afresh
            st = lib.rwkvb_batch_decode_greedy(h, 1, optr, s)
            assert st == native.RWKVB_ETIMEOUT, lib.rwkvb_status_string(st).decode()
            torch.cuda.synchronize(dev)  # no sticky CUDA error
        finally:
            lib.rwkvb_batch_destroy(h)
        # the context is intact: an ordinary engine on the same device decodes
        eng = B200BatchEngine(pack, nb, device=dev)
        try:
            eng.forward([3, 5])
            ids = eng.decode_greedy(2)
            assert ids.shape == (2, nb)
        finally:
            eng.close()


def test_status_string_names_timeout():
    assert "time" in native.lib().rwkvb_status_string(native.RWKVB_ETIMEOUT).decode().lower()
    with pytest.raises(RwkvbError):
        native.check(native.RWKVB_ETIMEOUT, "probe")
