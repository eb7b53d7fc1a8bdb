"""Pin the CPU oracle against vectors produced by the reference itself.

The fixtures in ``tests/golden`` come from the reference engine's encoders,
its C kernels built from source and its packed RWKV-7 forward
(``tests/golden/make_golden.py``).  Codec results must be bit-exact; GEMV
results match to the reference tests' own tolerance (1e-5,
``tests/test_grouped_fused_gemv.py:40-71`` in the reference), since the
restatement is scalar where the reference uses AVX2 reductions.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import cases, load_golden
from oracle import codec as oc
from oracle import kernels as ok
from oracle.forward import OracleRWKV7
from rwkv_b200 import synth

SG8 = load_golden("codec_sg8.npz")
LUT2 = load_golden("codec_lut2.npz")
GEMV = load_golden("gemv.npz")


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("case", cases(SG8))
def test_sg8_encode_decode_bit_exact(case):
    x = SG8[f"{case}/input"]
    g = int(SG8[f"{case}/group"])
    blob = SG8[f"{case}/blob"].tobytes()
    assert oc.encode_sg8(x, g) == blob
    dec = oc.decode_sg8(blob, x.size)
    assert np.array_equal(_bits(dec), _bits(SG8[f"{case}/decoded"].reshape(-1)))


@pytest.mark.parametrize("case", cases(SG8))
def test_product_sg8_encoder_matches_reference_bytes(case):
    x = torch.from_numpy(SG8[f"{case}/input"])
    g = int(SG8[f"{case}/group"])
    assert synth.encode_sg8(x, g).numpy().tobytes() == SG8[f"{case}/blob"].tobytes()


@pytest.mark.parametrize("case", cases(LUT2))
def test_lut2_decode_bit_exact(case):
    blob = LUT2[f"{case}/blob"].tobytes()
    x = LUT2[f"{case}/input"]
    dec = oc.decode_lut2_grouped(blob, x.shape)
    assert np.array_equal(_bits(dec), _bits(LUT2[f"{case}/decoded"]))


@pytest.mark.parametrize("case", [c for c in cases(LUT2) if c.startswith(("kmeans_fp16", "kmeans_fp32", "input_fp16"))])
def test_lut2_encode_bit_exact(case):
    x = LUT2[f"{case}/input"]
    g = int(LUT2[f"{case}/group"])
    kind = {"kmeans_fp16": oc.LUT2_GROUPED_FP16, "kmeans_fp32": oc.LUT2_GROUPED,
            "input_fp16": oc.LUT2_INPUT_FP16}[case.rsplit("_", 2)[0]]
    assert oc.encode_lut2_grouped(x, g, kind=kind) == LUT2[f"{case}/blob"].tobytes()


def test_product_lut2_encoder_is_a_valid_tr2_04_pack():
    """The torch LUT2 encoder (used to make large benchmark packs) writes the
    ``TR2\\x04`` layout and reaches k-means quality comparable to the
    reference encoder's."""
    case = "kmeans_fp16_64x128_g64"
    x = LUT2[f"{case}/input"]
    ref_blob = LUT2[f"{case}/blob"].tobytes()
    got = synth.encode_lut2(torch.from_numpy(x), 64).numpy().tobytes()
    assert got[:8] == ref_blob[:8] and len(got) == len(ref_blob)
    err_ref = np.abs(oc.decode_lut2_grouped(ref_blob, x.shape) - x).mean()
    err_got = np.abs(oc.decode_lut2_grouped(got, x.shape) - x).mean()
    assert err_got <= err_ref * 1.05


@pytest.mark.parametrize("impl", ["oracle", "reference"])
def test_gemv_family_matches_reference_kernels(impl):
    if impl == "reference" and not ok.ref_available():
        pytest.skip("reference C kernels not built")
    tol = dict(rtol=1e-5, atol=1e-5)
    for c in cases(GEMV):
        d = {k.split("/", 1)[1]: v for k, v in GEMV.items() if k.startswith(c + "/")}
        if c.startswith("sg8_"):
            o, i = d["shape"]
            np.testing.assert_allclose(ok.sg8_gemv(d["blob"], d["x"], o, i, impl), d["y"], **tol, err_msg=c)
        elif c.startswith("lut2_"):
            o, i = d["shape"]
            np.testing.assert_allclose(ok.lut2_gemv(d["blob"], d["x"], o, i, impl), d["y"], **tol, err_msg=c)
        elif c.startswith("tr_"):
            i, o = d["shape"]
            np.testing.assert_allclose(ok.sg8_transposed_gemv(d["blob"], d["x"], o, i, impl), d["y"],
                                       **tol, err_msg=c)
        elif c.startswith("adapters_"):
            has_v = c.endswith("1")
            names = ["w1", "w2", "a1", "a2", "g1", "g2"] + (["v1", "v2"] if has_v else [])
            xs = [d[f"x{j}"] for j in range(4 if has_v else 3)]
            w, a, g, v = ok.sg8_tmix_adapters([d[f"blob_{n}"] for n in names], xs, d["a0"], 256,
                                              list(d["ranks"]), impl)
            for nm, got in (("w", w), ("a", a), ("g", g)) + ((("v", v),) if has_v else ()):
                np.testing.assert_allclose(got, d[nm], **tol, err_msg=f"{c}/{nm}")
        elif c == "cmix":
            ko, ki, vo, vi = d["dims"]
            np.testing.assert_allclose(ok.sg8_cmix(d["key_blob"], d["value_blob"], d["x"], ko, ki, vo, vi, impl),
                                       d["y"], rtol=1e-6, atol=1e-4, err_msg=c)
        elif c == "qkv":
            y = ok.sg8_tmix_qkv([d[f"blob{j}"] for j in range(3)], [d[f"x{j}"] for j in range(3)], 256, 256, impl)
            np.testing.assert_allclose(y, d["y"], **tol, err_msg=c)


def _oracle_pack(policy: str, gold: dict):
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
        if codec != "none":
            want = str(gold[f"sha256/{name}"])
            assert hashlib.sha256(payload).hexdigest() == want, f"encoder drift on {name}"
        pack[name] = synth.PackedTensor(name, tuple(t.shape), codec, payload)
    return shape, pack


@pytest.mark.parametrize("policy", ["sg8", "lut2"])
def test_oracle_forward_matches_reference_forward(policy):
    gold = load_golden(f"forward_tiny_{policy}.npz")
    shape, pack = _oracle_pack(policy, gold)
    model = OracleRWKV7(pack, n_layer=shape.n_layer, n_embd=shape.n_embd, head_size=shape.head_size)
    ids, logits, state = model.greedy([int(t) for t in gold["prompt"]], len(gold["ids"]))
    assert ids == [int(t) for t in gold["ids"]]
    np.testing.assert_allclose(logits, gold["logits"], rtol=0, atol=1e-4)
    for j, s in enumerate(state):
        np.testing.assert_allclose(s, gold[f"state/{j}"], rtol=0, atol=1e-4)


EXTRA = load_golden("gemv_extra.npz")


@pytest.mark.parametrize("impl", ["oracle", "reference"])
def test_per_tensor_lut2_and_int8_activation_match_reference_kernels(impl):
    """Legacy per-tensor LUT2 (``TR2\\x01``: decode K1, row-walk GEMV K3) and the
    activation-INT8 SG8 GEMV (K7) against the reference's own outputs."""
    if impl == "reference" and not ok.ref_available():
        pytest.skip("reference C kernels not built")
    for t in ("sq", "lin", "odd"):
        o, i = (int(v) for v in EXTRA[f"tensor_{t}/shape"])
        blob = EXTRA[f"tensor_{t}/blob"]
        y = ok.lut2_tensor_gemv(blob, EXTRA[f"tensor_{t}/x"], o, i, impl)
        np.testing.assert_allclose(y, EXTRA[f"tensor_{t}/y"], rtol=1e-5, atol=1e-6, err_msg=t)
        dec = oc.decode_lut2_tensor(blob.tobytes(), o * i)
        assert np.array_equal(dec.view(np.uint32), EXTRA[f"tensor_{t}/decoded"].reshape(-1).view(np.uint32)), t
    for t in ("sq", "g64"):
        o, i = (int(v) for v in EXTRA[f"i8_{t}/shape"])
        y = ok.sg8_i8_gemv(EXTRA[f"i8_{t}/blob"], EXTRA[f"i8_{t}/x"], o, i, impl)
        np.testing.assert_allclose(y, EXTRA[f"i8_{t}/y"], rtol=1e-5, atol=1e-6, err_msg=t)


def test_residual_and_per_tensor_encoders_round_trip():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((32, 128)) * 0.02).astype(np.float32)
    errs = {}
    for kind in oc.LUT2_GROUPED_KINDS:
        d = oc.decode_lut2_grouped(oc.encode_lut2_grouped(w, 64, kind=kind), w.shape)
        errs[kind] = float(np.abs(d - w).max())
    # two exact-ish residuals per group only lower the error
    assert errs[oc.LUT2_GROUPED_RESIDUAL] < errs[oc.LUT2_GROUPED_FP16]
    assert errs[oc.LUT2_INPUT_RESIDUAL] < errs[oc.LUT2_INPUT_FP16]
    d = oc.decode_lut2_tensor(oc.encode_lut2_tensor(w), w.size)
    assert float(np.abs(d.reshape(w.shape) - w).max()) < 0.1
