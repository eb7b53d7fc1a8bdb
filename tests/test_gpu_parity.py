"""GPU parity: the sm_100a library (through its C ABI) against the oracle and
the reference-generated golden vectors.

Bars (from the engine's contract):
* dequantised weights: bit-exact;
* packed GEMV family: rtol/atol 2e-5 against the reference C kernels (fp32,
  different reduction order);
* full decode: greedy ids identical, logits and recurrent state within 1e-3
  max-abs (the contract allows 1e-2).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cases, load_golden

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU-only hosts
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle import codec as oc  # noqa: E402
from oracle import kernels as ok  # noqa: E402
from oracle.forward import OracleRWKV7  # noqa: E402
from rwkv_b200 import lut_gemm_fused as lg  # noqa: E402
from rwkv_b200 import synth  # noqa: E402
from rwkv_b200.engine import B200Engine  # noqa: E402

TOL = dict(rtol=2e-5, atol=2e-5)
LOGIT_TOL = 1e-3


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("fixture", ["codec_sg8.npz", "codec_lut2.npz"])
def test_device_dequant_bit_exact(fixture):
    g = load_golden(fixture)
    for c in cases(g):
        x = g[f"{c}/input"]
        shape = x.shape if x.ndim == 2 else (1, x.size)
        got = lg.decode_packed(g[f"{c}/blob"].tobytes(), *shape)
        assert np.array_equal(_bits(_np(got).reshape(-1)), _bits(g[f"{c}/decoded"].reshape(-1))), c


def test_gemv_family_matches_reference_kernels():
    G = load_golden("gemv.npz")
    for c in cases(G):
        d = {k.split("/", 1)[1]: v for k, v in G.items() if k.startswith(c + "/")}
        if c.startswith(("sg8_", "lut2_")):
            o, i = (int(v) for v in d["shape"])
            y = lg.lut2_gemv(d["blob"].tobytes(), torch.from_numpy(d["x"]), out_features=o, in_features=i)
            # the reference LUT2 kernel sums sequentially in fp32 (lut2_gather.c:300-324): its own
            # rounding error reaches ~1e-4 relative on these rows
            tol = TOL if c.startswith("sg8_") else dict(rtol=1e-4, atol=1e-4)
            np.testing.assert_allclose(_np(y), d["y"], **tol, err_msg=c)
        elif c.startswith("tr_"):
            i, o = (int(v) for v in d["shape"])
            y = lg.grouped_u8_transposed_gemv(d["blob"].tobytes(), torch.from_numpy(d["x"]), out_features=o,
                                              in_features=i)
            np.testing.assert_allclose(_np(y), d["y"], **TOL, err_msg=c)
        elif c.startswith("adapters_"):
            has_v = c.endswith("1")
            names = ["w1", "w2", "a1", "a2", "g1", "g2"] + (["v1", "v2"] if has_v else [])
            rw, ra, rg, rv = (int(v) for v in d["ranks"])
            rk = {"w": rw, "a": ra, "g": rg, "v": rv}
            shapes = [((256, rk[n[0]]) if n.endswith("1") else (rk[n[0]], 256)) for n in names]
            xs = [torch.from_numpy(d[f"x{j}"]) for j in range(4 if has_v else 3)]
            res = lg.grouped_u8_transposed_tmix_fused([d[f"blob_{n}"].tobytes() for n in names], xs, shapes,
                                                      torch.from_numpy(d["a0"]))
            for nm, got in zip(("w", "a", "g", "v"), res):
                np.testing.assert_allclose(_np(got), d[nm], **TOL, err_msg=f"{c}/{nm}")
        elif c == "cmix":
            ko, ki, vo, vi = (int(v) for v in d["dims"])
            y = lg.grouped_u8_cmix_gemv(d["key_blob"].tobytes(), d["value_blob"].tobytes(), torch.from_numpy(d["x"]),
                                        key_out_features=ko, key_in_features=ki, value_out_features=vo,
                                        value_in_features=vi)
            np.testing.assert_allclose(_np(y), d["y"], rtol=1e-5, atol=1e-4, err_msg=c)
        elif c == "qkv":
            ys = lg.lut2_tmix_qkv_gemv_batched([d[f"blob{j}"].tobytes() for j in range(3)],
                                               [torch.from_numpy(d[f"x{j}"]) for j in range(3)],
                                               out_features=256, in_features=256)
            np.testing.assert_allclose(np.stack([_np(y) for y in ys]), d["y"], **TOL, err_msg=c)


@pytest.mark.parametrize("shape,g", [((10240, 2560), 128), ((2560, 10240), 128), ((2560, 2560), 64)])
def test_sg8_gemv_full_size_matches_oracle(shape, g):
    """2.9B-config projection shapes (fast vectorised path) against the oracle C GEMV."""
    gen = torch.Generator().manual_seed(shape[0] + g)
    w = torch.randn(shape, generator=gen) * 0.02
    x = torch.randn(shape[1], generator=gen)
    blob = synth.encode_sg8(w.cuda(), g).cpu().numpy().tobytes()
    dec = oc.decode_sg8(blob, shape[0] * shape[1]).reshape(shape).astype(np.float64)
    exact = dec @ x.numpy().astype(np.float64)
    got = lg.lut2_gemv(blob, x, out_features=shape[0], in_features=shape[1])
    np.testing.assert_allclose(_np(got), exact, rtol=2e-5, atol=2e-5)
    # the oracle's sequential fp32 sum is the looser of the two
    np.testing.assert_allclose(ok.sg8_gemv(blob, x.numpy(), shape[0], shape[1]), exact, rtol=1e-3, atol=1e-3)
    # dequant of the same blob stays bit-exact at full size
    dq = lg.decode_packed(blob, *shape)
    assert np.array_equal(_bits(_np(dq).reshape(-1)), _bits(oc.decode_sg8(blob, shape[0] * shape[1])))


def test_lut2_gemv_full_size_matches_oracle():
    gen = torch.Generator().manual_seed(5)
    w = torch.randn((2560, 2560), generator=gen) * 0.02
    x = torch.randn(2560, generator=gen)
    blob = synth.encode_lut2(w.cuda(), 64).cpu().numpy().tobytes()
    exact = oc.decode_lut2_grouped(blob, (2560, 2560)).astype(np.float64) @ x.numpy().astype(np.float64)
    got = lg.lut2_gemv(blob, x, out_features=2560, in_features=2560)
    np.testing.assert_allclose(_np(got), exact, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(ok.lut2_gemv(blob, x.numpy(), 2560, 2560), exact, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("decay_mode", [0, 1])
def test_wkv7_op_matches_numpy(decay_mode):
    B, H, N = 2, 3, 64
    gen = torch.Generator().manual_seed(11 + decay_mode)
    S = torch.randn((B, H, N, N), generator=gen) * 0.1
    r, w, k, v, a = (torch.randn((B, H * N), generator=gen) for _ in range(5))
    kk = torch.nn.functional.normalize(torch.randn((B, H, N), generator=gen), dim=-1).reshape(B, H * N)
    a = torch.sigmoid(a)
    d = torch.exp(-0.606531 * torch.sigmoid(w)) if decay_mode == 0 else torch.exp(-torch.exp(w))
    Sn = S.numpy().astype(np.float64)
    rr, dd, kv, vv, kkv, aa = (t.reshape(B, H, N).numpy().astype(np.float64) for t in (r, d, k, v, kk, a))
    sa = np.einsum("bhij,bhj->bhi", Sn, -kkv)
    Sn = Sn * dd[:, :, None, :] + sa[..., None] * (kkv * aa)[:, :, None, :] + vv[..., None] * kv[:, :, None, :]
    y_ref = np.einsum("bhij,bhj->bhi", Sn, rr).reshape(B, H * N)
    Sd = S.cuda().contiguous()
    y = lg.wkv7(Sd, r, w, k, v, kk, a, decay_mode=decay_mode)
    np.testing.assert_allclose(_np(y), y_ref, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(_np(Sd), Sn, rtol=1e-4, atol=1e-4)


def _reference_pack(policy: str):
    gold = load_golden(f"forward_tiny_{policy}.npz")
    shape = synth.PRESETS["tiny"]
    sd = synth.generate_state_dict(shape, int(gold["seed"]), "cpu")
    pack = {}
    for name, t in sd.items():
        codec = synth.codec_for(name, tuple(t.shape), policy)
        arr = t.numpy()
        if codec == "none":
            payload = arr.reshape(-1).copy()
        elif codec == "sg8":
            payload = oc.encode_sg8(arr, 128)
        else:
            payload = oc.encode_lut2_grouped(arr, 64, kind=oc.LUT2_GROUPED_FP16)
        pack[name] = synth.PackedTensor(name, tuple(t.shape), codec, payload)
    return gold, shape, pack


@pytest.mark.parametrize("policy", ["sg8", "lut2"])
@pytest.mark.parametrize("path", ["persistent", "graph", "nograph"])
def test_engine_decode_matches_reference_forward(policy, path):
    gold, shape, pack = _reference_pack(policy)
    eng = B200Engine(pack, use_graph=path != "nograph", persistent=path == "persistent")
    try:
        # SG8 packs run the persistent kernel when asked; LUT2 packs always use the graph path
        assert eng.persistent_active == (path == "persistent" and policy == "sg8")
        prompt = [int(t) for t in gold["prompt"]]
        ids, logits = eng.greedy(prompt, len(gold["ids"]), keep_logits=True)
        assert ids == [int(t) for t in gold["ids"]]
        np.testing.assert_allclose(_np(logits), gold["logits"], rtol=0, atol=LOGIT_TOL)
        st = eng.get_state()
        for j, s in enumerate(st):
            np.testing.assert_allclose(_np(s).reshape(-1), gold[f"state/{j}"].reshape(-1), rtol=0, atol=LOGIT_TOL)
        # the on-device greedy loop (no host round trip per token) gives the same ids
        eng.reset()
        ids2, _ = eng.greedy(prompt, len(gold["ids"]))
        assert ids2 == ids
    finally:
        eng.close()


def test_engine_ffn_row_order_matches_reference_forward():
    """The persistent kernel with the FFN value units in row order and fp32
    accumulation (the default orders them by column chunk and sums in fixed
    point): same ids, logits and state as the reference forward."""
    gold, shape, pack = _reference_pack("sg8")
    eng = B200Engine(pack, ffn_chunk_order=False)
    try:
        assert eng.persistent_active
        ids, logits = eng.greedy([int(t) for t in gold["prompt"]], len(gold["ids"]), keep_logits=True)
        assert ids == [int(t) for t in gold["ids"]]
        np.testing.assert_allclose(_np(logits), gold["logits"], rtol=0, atol=LOGIT_TOL)
        for j, st in enumerate(eng.get_state()):
            np.testing.assert_allclose(_np(st).reshape(-1), gold[f"state/{j}"].reshape(-1), rtol=0, atol=LOGIT_TOL)
    finally:
        eng.close()


@pytest.mark.parametrize("prefetch", [0, 1, 2])
def test_engine_prefetch_distance_does_not_change_results(prefetch):
    gold, shape, pack = _reference_pack("sg8")
    eng = B200Engine(pack, prefetch_distance=prefetch)
    try:
        ids, _ = eng.greedy([int(t) for t in gold["prompt"]], len(gold["ids"]))
        assert ids == [int(t) for t in gold["ids"]]
    finally:
        eng.close()


def test_engine_state_roundtrip_and_reset():
    gold, shape, pack = _reference_pack("sg8")
    eng = B200Engine(pack)
    try:
        prompt = [int(t) for t in gold["prompt"]]
        eng.forward(prompt)
        snap = eng.get_state()
        first = int(torch.argmax(eng.logits))
        a = eng.decode_greedy(first, 6)
        eng.set_state(snap)
        b = eng.decode_greedy(first, 6)
        assert a == b
        eng.reset()
        assert float(eng.wkv.abs().sum()) == 0.0
    finally:
        eng.close()


def test_engine_rejects_out_of_range_token():
    from rwkv_b200.native import RwkvbError

    _, shape, pack = _reference_pack("sg8")
    eng = B200Engine(pack)
    try:
        with pytest.raises(RwkvbError):
            eng.forward([shape.vocab])
        with pytest.raises(RwkvbError):
            eng.decode_greedy(-1, 2)
    finally:
        eng.close()


@pytest.mark.parametrize("persistent", [True, False])
def test_engine_0p1b_shape_matches_oracle_first_tokens(persistent):
    """Real 0.1B dimensions (12 layers, d_model 768, vocab 65536), seeded weights:
    the first decode steps against the oracle forward."""
    shape = synth.PRESETS["0.1b"]
    sd = synth.generate_state_dict(shape, 3, "cpu")
    pack = synth.make_pack(sd, policy="sg8")
    model = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    prompt = synth.seeded_prompt(3, shape.vocab, 3)
    ids_ref, logits_ref, state_ref = model.greedy(prompt, 3)
    eng = B200Engine(pack, persistent=persistent)
    try:
        assert eng.persistent_active == persistent
        ids, logits = eng.greedy(prompt, 3, keep_logits=True)
        assert ids == ids_ref
        np.testing.assert_allclose(_np(logits), logits_ref, rtol=0, atol=LOGIT_TOL)
        st = eng.get_state()
        for j in range(0, len(st), 7):
            np.testing.assert_allclose(_np(st[j]).reshape(-1), state_ref[j].reshape(-1), rtol=0, atol=LOGIT_TOL)
    finally:
        eng.close()


def test_per_tensor_lut2_int8_activation_and_four_maps_match_reference_kernels():
    """``gemv_extra.npz`` (reference encoders and C kernels): per-tensor LUT2
    decode bit-exact (K1), its row-walk GEMV (K3), the four/three-map batches
    (K15, K13), the activation-INT8 SG8 GEMV (K7) and its QKV maps (K14)."""
    E = load_golden("gemv_extra.npz")
    for t in ("sq", "lin", "odd"):
        o, i = (int(v) for v in E[f"tensor_{t}/shape"])
        blob = E[f"tensor_{t}/blob"].tobytes()
        got = _np(lg.decode_packed(blob, o, i)).reshape(-1)
        assert np.array_equal(_bits(got), _bits(E[f"tensor_{t}/decoded"].reshape(-1))), t
        y = lg.lut2_gemv(blob, torch.from_numpy(E[f"tensor_{t}/x"]), out_features=o, in_features=i)
        np.testing.assert_allclose(_np(y), E[f"tensor_{t}/y"], **TOL, err_msg=t)
    C = 128
    blobs = [E[f"tensor_maps/blob{j}"].tobytes() for j in range(4)]
    xs = [torch.from_numpy(E[f"tensor_maps/x{j}"]) for j in range(4)]
    ys = lg.lut2_tmix_gemv_batched(blobs, xs, out_features=C, in_features=C)
    np.testing.assert_allclose(np.stack([_np(y) for y in ys]), E["tensor_maps/y4"], **TOL)
    ys = lg.lut2_tmix_qkv_gemv_batched(blobs[:3], xs[:3], out_features=C, in_features=C)
    np.testing.assert_allclose(np.stack([_np(y) for y in ys]), E["tensor_maps/y3"], **TOL)
    blobs = [E[f"sg8_maps/blob{j}"].tobytes() for j in range(4)]
    xs = [torch.from_numpy(E[f"sg8_maps/x{j}"]) for j in range(4)]
    ys = lg.lut2_tmix_gemv_batched(blobs, xs, out_features=C, in_features=2 * C)
    np.testing.assert_allclose(np.stack([_np(y) for y in ys]), E["sg8_maps/y4"], **TOL)
    for t in ("sq", "g64"):
        o, i = (int(v) for v in E[f"i8_{t}/shape"])
        y = lg.lut2_gemv(E[f"i8_{t}/blob"].tobytes(), torch.from_numpy(E[f"i8_{t}/x"]), out_features=o,
                         in_features=i, activation_int8=True)
        np.testing.assert_allclose(_np(y), E[f"i8_{t}/y"], **TOL, err_msg=t)
    import os

    os.environ["RWKV_LUT_ACTIVATION_INT8"] = "1"
    try:
        blobs = [E[f"i8_qkv/blob{j}"].tobytes() for j in range(3)]
        xs = [torch.from_numpy(E[f"i8_qkv/x{j}"]) for j in range(3)]
        ys = lg.lut2_tmix_qkv_gemv_batched(blobs, xs, out_features=C, in_features=2 * C)
    finally:
        os.environ["RWKV_LUT_ACTIVATION_INT8"] = "0"
    np.testing.assert_allclose(np.stack([_np(y) for y in ys]), E["i8_qkv/y"], **TOL)


def _kind_pack(kind: bytes, seed: int):
    """The tiny model with its projections and head in one LUT2 wire kind
    (``TR2\\x01`` per-tensor, or a grouped kind 3..7), adapters / embedding SG8."""
    shape = synth.PRESETS["tiny"]
    sd = synth.generate_state_dict(shape, seed, "cpu")
    pack = {}
    for name, t in sd.items():
        arr = t.numpy()
        codec = synth.codec_for(name, tuple(t.shape), "lut2")
        if codec == "none":
            pack[name] = synth.PackedTensor(name, tuple(t.shape), "none", arr.reshape(-1).copy())
        elif codec == "sg8":
            pack[name] = synth.PackedTensor(name, tuple(t.shape), "sg8", oc.encode_sg8(arr, 128))
        else:
            blob = oc.encode_lut2_tensor(arr) if kind == b"TR2\x01" else oc.encode_lut2_grouped(arr, 64, kind=kind)
            pack[name] = synth.PackedTensor(name, tuple(t.shape), "lut2", blob)
    return shape, pack


@pytest.mark.parametrize("kind", [b"TR2\x01", oc.LUT2_GROUPED, oc.LUT2_GROUPED_RESIDUAL, oc.LUT2_INPUT_FP16,
                                  oc.LUT2_INPUT_RESIDUAL])
def test_engine_decodes_every_lut2_wire_kind_like_the_oracle(kind):
    """The batch-1 engine on packs whose projections and head use each LUT2
    wire kind (the multi-kernel step) against the oracle forward."""
    shape, pack = _kind_pack(kind, 17 + kind[3])
    model = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    prompt = synth.seeded_prompt(4, shape.vocab, 17)
    ids_ref, logits_ref, state_ref = model.greedy(prompt, 6)
    eng = B200Engine(pack)
    try:
        ids, logits = eng.greedy(prompt, 6, keep_logits=True)
        assert ids == ids_ref
        np.testing.assert_allclose(_np(logits), logits_ref, rtol=0, atol=LOGIT_TOL)
        for j, s in enumerate(eng.get_state()):
            np.testing.assert_allclose(_np(s).reshape(-1), state_ref[j].reshape(-1), rtol=0, atol=LOGIT_TOL)
    finally:
        eng.close()
