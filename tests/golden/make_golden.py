"""Generate golden vectors from the reference engine itself.

Runs ONLY in the development container, where the reference source tree is
mounted read-only at ``/root/reference`` (override with ``RWKV_REF_ROOT``).
The reference package is copied to a temporary directory, its
``lut2_gather.c`` is compiled there from source (same recipe as
``oracle/Makefile``), and the reference's own Python and C code produce:

* ``codec_sg8.npz``    — ``encode_scale_u8_grouped`` blobs + ``decode_scale_u8_grouped_to_tensor`` values
* ``codec_lut2.npz``   — ``encode_trinity_lut2`` blobs (kinds 3..7) + decoded values
* ``gemv.npz``         — outputs of the reference C kernels (SG8 / LUT2 / transposed /
                         fused adapters / fused CMix / batched QKV)
* ``gemv_extra.npz``   — legacy per-tensor LUT2 (``TR2\\x01``) decode / GEMV / batched maps,
                         four-map SG8 batch, activation-INT8 SG8 GEMV and QKV maps
* ``forward_tiny_sg8.npz`` / ``forward_tiny_lut2.npz`` — the reference packed RWKV-7 forward
  (``forward_block_packed`` + packed head + argmax) on the seeded 4-layer, d_model 256 model:
  8 prompt tokens then 16 greedy tokens; per-pass logits, ids and final recurrent state,
  plus the sha256 of every packed blob.

The committed ``.npz`` files are what the tests read; nothing at test time
touches the reference tree.  Re-run with::

    python tests/golden/make_golden.py [codec] [gemv] [extra] [forward]   # default: all
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF_ROOT = Path(os.environ.get("RWKV_REF_ROOT", "/root/reference"))

SEED = 1234
PROMPT_LEN = 8
GEN_LEN = 16


def _prepare_reference() -> Path:
    tmp = Path(tempfile.mkdtemp(prefix="rwkv_ref_"))
    shutil.copytree(REF_ROOT / "rwkv_ssd", tmp / "rwkv_ssd",
                    ignore=shutil.ignore_patterns("*.dll", "__pycache__"))
    subprocess.run(["/usr/bin/gcc", "-shared", "-O3", "-mavx2", "-mfma", "-fPIC", "-fopenmp",
                    "-o", str(tmp / "rwkv_ssd/native/lut2_gather.so"),
                    str(REF_ROOT / "rwkv_ssd/native/lut2_gather.c")], check=True)
    sys.path.insert(0, str(tmp))
    return tmp


def _entry(name, shape, length, codec):
    from rwkv_ssd.runtime.manifest import TensorEntry
    return TensorEntry(name=name, layer_id=0, dtype="float32", shape=list(shape), offset=0,
                       length=length, alignment=1, residency="streamed", dequant=codec)


def _sha(b: bytes) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def codec_fixtures() -> None:
    from rwkv_ssd.runtime.pack_codec import decode_scale_u8_grouped_to_tensor, encode_scale_u8_grouped
    from rwkv_ssd.runtime.trinity_codec import decode_trinity_lut2_to_tensor, encode_trinity_lut2

    gen = torch.Generator().manual_seed(SEED)
    sg8_cases = [
        ("matrix_g128", (64, 256), 128, "normal"),
        ("ragged_rows_g64", (96, 200), 64, "normal"),
        ("adapter_straddle_g128", (256, 96), 128, "normal"),
        ("tiny_g4", (7, 5), 4, "normal"),
        ("partial_tail_g128", (1000,), 128, "normal"),
        ("outliers_g128", (32, 256), 128, "outlier"),
        ("constant_groups_g128", (4, 256), 128, "const"),
        ("single_value", (1,), 128, "normal"),
    ]
    out: dict[str, np.ndarray] = {}
    for name, shape, g, kind in sg8_cases:
        t = torch.randn(shape, generator=gen) * 0.02
        if kind == "outlier":
            t.view(-1)[::97] *= 400.0
        if kind == "const":
            t = torch.full(shape, 0.25)
            t[1] = -3.0
            t[2, :128] = torch.linspace(-1, 1, 128)
        blob = encode_scale_u8_grouped(t, group_size=g)
        dec = decode_scale_u8_grouped_to_tensor(blob, _entry(name, shape, len(blob), "scale_u8_grouped"),
                                                torch.device("cpu"))
        out[f"{name}/input"] = t.numpy().astype(np.float32)
        out[f"{name}/group"] = np.array(g)
        out[f"{name}/blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"{name}/decoded"] = dec.numpy().astype(np.float32)
    np.savez_compressed(HERE / "codec_sg8.npz", **out)

    out = {}
    algos = [("kmeans_fp32", "groupwise_kmeans"), ("kmeans_fp16", "groupwise_kmeans_fp16"),
             ("kmeans_residual", "groupwise_kmeans_residual"), ("input_fp16", "groupwise_input_fp16"),
             ("input_residual", "groupwise_input_residual")]
    for shape, g in (((7, 5), 4), ((64, 128), 64), ((33, 40), 64)):
        t = torch.randn(shape, generator=gen) * 0.02
        for tag, algo in algos:
            key = f"{tag}_{shape[0]}x{shape[1]}_g{g}"
            blob = encode_trinity_lut2(t, codebook=algo, group_size=g)
            dec = decode_trinity_lut2_to_tensor(blob, _entry(key, shape, len(blob), "trinity_lut2"),
                                                torch.device("cpu"))
            out[f"{key}/input"] = t.numpy().astype(np.float32)
            out[f"{key}/group"] = np.array(g)
            out[f"{key}/blob"] = np.frombuffer(blob, np.uint8).copy()
            out[f"{key}/decoded"] = dec.float().numpy().astype(np.float32)
    np.savez_compressed(HERE / "codec_lut2.npz", **out)


def gemv_fixtures() -> None:
    os.environ["RWKV_LUT_KERNEL"] = "c"
    from rwkv_ssd.runtime import lut_gemm_fused as lg
    from rwkv_ssd.runtime.pack_codec import encode_scale_u8_grouped
    from rwkv_ssd.runtime.trinity_codec import encode_trinity_lut2

    gen = torch.Generator().manual_seed(SEED + 1)
    out: dict[str, np.ndarray] = {}

    def rnd(*s, scale=0.02):
        return torch.randn(s, generator=gen) * scale

    # SG8 W @ x (K5)
    for tag, (o, i), g in (("sq", (256, 256), 128), ("tall", (512, 128), 128),
                           ("ragged", (96, 200), 64), ("tiny", (7, 5), 4)):
        w, x = rnd(o, i), rnd(i, scale=1.0)
        blob = encode_scale_u8_grouped(w, group_size=g)
        y = lg.lut2_gemv(blob, x, out_features=o, in_features=i)
        out[f"sg8_{tag}/blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"sg8_{tag}/x"] = x.numpy()
        out[f"sg8_{tag}/y"] = y.numpy()
        out[f"sg8_{tag}/shape"] = np.array([o, i])
    # grouped LUT2 W @ x (K4), every kind
    os.environ["RWKV_LUT_KERNEL"] = "auto"
    for algo in ("groupwise_kmeans", "groupwise_kmeans_fp16", "groupwise_kmeans_residual",
                 "groupwise_input_fp16", "groupwise_input_residual"):
        for tag, (o, i), g in (("sq", (128, 256), 64), ("ragged", (33, 40), 64)):
            w, x = rnd(o, i), rnd(i, scale=1.0)
            blob = encode_trinity_lut2(w, codebook=algo, group_size=g)
            y = lg.lut2_gemv(blob, x, out_features=o, in_features=i)
            key = f"lut2_{algo}_{tag}"
            out[f"{key}/blob"] = np.frombuffer(blob, np.uint8).copy()
            out[f"{key}/x"] = x.numpy()
            out[f"{key}/y"] = y.numpy()
            out[f"{key}/shape"] = np.array([o, i])
    os.environ["RWKV_LUT_KERNEL"] = "c"
    # transposed x @ W (K8), W row-major [in, out]
    for tag, (i, o), g in (("w1", (256, 32), 128), ("w2", (32, 256), 128), ("g1", (256, 64), 128),
                           ("straddle", (200, 96), 128)):
        w, x = rnd(i, o), rnd(i, scale=1.0)
        blob = encode_scale_u8_grouped(w, group_size=g)
        y = lg.grouped_u8_transposed_gemv(blob, x, out_features=o, in_features=i)
        out[f"tr_{tag}/blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"tr_{tag}/x"] = x.numpy()
        out[f"tr_{tag}/y"] = y.numpy()
        out[f"tr_{tag}/shape"] = np.array([i, o])
    # fused adapters (K10), with and without the v pair
    C, rw, ra, rv, rg = 256, 32, 32, 32, 64
    for has_v in (False, True):
        mats = {"w1": rnd(C, rw), "w2": rnd(rw, C), "a1": rnd(C, ra), "a2": rnd(ra, C),
                "g1": rnd(C, rg), "g2": rnd(rg, C), "v1": rnd(C, rv), "v2": rnd(rv, C)}
        names = ["w1", "w2", "a1", "a2", "g1", "g2"] + (["v1", "v2"] if has_v else [])
        blobs = tuple(encode_scale_u8_grouped(mats[n], group_size=128) for n in names)
        xs = tuple(torch.rand(C, generator=gen) for _ in range(4 if has_v else 3))
        a0 = torch.rand(C, generator=gen) * 2 - 1
        shapes = tuple(tuple(mats[n].shape) for n in names)
        res = lg.grouped_u8_transposed_tmix_fused(blobs, xs, shapes, a0)
        key = f"adapters_v{int(has_v)}"
        for n, b in zip(names, blobs):
            out[f"{key}/blob_{n}"] = np.frombuffer(b, np.uint8).copy()
        for j, xx in enumerate(xs):
            out[f"{key}/x{j}"] = xx.numpy()
        out[f"{key}/a0"] = a0.numpy()
        out[f"{key}/ranks"] = np.array([rw, ra, rg, rv if has_v else 0])
        for n, r in zip(("w", "a", "g", "v"), res):
            out[f"{key}/{n}"] = r.numpy()
    # fused CMix (K6)
    F = 1024
    wk, wv, x = rnd(F, C), rnd(C, F), torch.rand(C, generator=gen) * 2 - 1
    kb = encode_scale_u8_grouped(wk, group_size=128)
    vb = encode_scale_u8_grouped(wv, group_size=128)
    y = lg.grouped_u8_cmix_gemv(kb, vb, x, key_out_features=F, key_in_features=C,
                                value_out_features=C, value_in_features=F)
    out["cmix/key_blob"] = np.frombuffer(kb, np.uint8).copy()
    out["cmix/value_blob"] = np.frombuffer(vb, np.uint8).copy()
    out["cmix/x"] = x.numpy()
    out["cmix/y"] = y.numpy()
    out["cmix/dims"] = np.array([F, C, C, F])
    # batched QKV (K13)
    blobs = tuple(encode_scale_u8_grouped(rnd(C, C), group_size=128) for _ in range(3))
    xs = tuple(rnd(C, scale=1.0) for _ in range(3))
    r, k, v = lg.lut2_tmix_qkv_gemv_batched(blobs, xs, out_features=C, in_features=C)
    for j, b in enumerate(blobs):
        out[f"qkv/blob{j}"] = np.frombuffer(b, np.uint8).copy()
        out[f"qkv/x{j}"] = xs[j].numpy()
    out["qkv/y"] = torch.stack([r, k, v]).numpy()
    np.savez_compressed(HERE / "gemv.npz", **out)


def extra_fixtures() -> None:
    """``gemv_extra.npz``: legacy per-tensor LUT2 ``TR2\\x01`` (decode K1, W @ x
    K3, four- and three-map batches K15), the four-map SG8 batch (K13) and the
    activation-INT8 SG8 kernels (K7, K14), all from the reference's own
    encoders and C kernels."""
    os.environ["RWKV_LUT_KERNEL"] = "c"
    from rwkv_ssd.runtime import lut_gemm_fused as lg
    from rwkv_ssd.runtime.pack_codec import encode_scale_u8_grouped
    from rwkv_ssd.runtime.trinity_codec import decode_trinity_lut2_to_tensor, encode_trinity_lut2

    gen = torch.Generator().manual_seed(SEED + 2)
    out: dict[str, np.ndarray] = {}

    def rnd(*s, scale=0.02):
        return torch.randn(s, generator=gen) * scale

    # TR2\x01: one fp32 codebook per tensor; "odd" has rows that do not start on
    # a code byte (the K3 row walk reads them from the row's first whole byte)
    for tag, (o, i), algo in (("sq", (64, 256), "kmeans"), ("lin", (48, 128), "linspace"),
                              ("odd", (9, 13), "kmeans")):
        w, x = rnd(o, i), rnd(i, scale=1.0)
        blob = encode_trinity_lut2(w, codebook=algo)
        assert bytes(blob[:4]) == b"TR2\x01"
        dec = decode_trinity_lut2_to_tensor(blob, _entry(tag, (o, i), len(blob), "trinity_lut2"),
                                            torch.device("cpu"))
        y = lg.lut2_gemv(blob, x, out_features=o, in_features=i)
        key = f"tensor_{tag}"
        out[f"{key}/blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"{key}/x"] = x.numpy()
        out[f"{key}/y"] = y.numpy()
        out[f"{key}/decoded"] = dec.float().numpy()
        out[f"{key}/shape"] = np.array([o, i])
    C = 128
    blobs = tuple(encode_trinity_lut2(rnd(C, C), codebook="kmeans") for _ in range(4))
    xs = tuple(rnd(C, scale=1.0) for _ in range(4))
    ys = lg.lut2_tmix_gemv_batched(blobs, xs, out_features=C, in_features=C)
    ys3 = lg.lut2_tmix_qkv_gemv_batched(blobs[:3], xs[:3], out_features=C, in_features=C)
    for j in range(4):
        out[f"tensor_maps/blob{j}"] = np.frombuffer(blobs[j], np.uint8).copy()
        out[f"tensor_maps/x{j}"] = xs[j].numpy()
    out["tensor_maps/y4"] = torch.stack(list(ys)).numpy()
    out["tensor_maps/y3"] = torch.stack(list(ys3)).numpy()
    # SG8 four maps (K13)
    blobs = tuple(encode_scale_u8_grouped(rnd(C, 2 * C), group_size=128) for _ in range(4))
    xs = tuple(rnd(2 * C, scale=1.0) for _ in range(4))
    ys = lg.lut2_tmix_gemv_batched(blobs, xs, out_features=C, in_features=2 * C)
    for j in range(4):
        out[f"sg8_maps/blob{j}"] = np.frombuffer(blobs[j], np.uint8).copy()
        out[f"sg8_maps/x{j}"] = xs[j].numpy()
    out["sg8_maps/y4"] = torch.stack(list(ys)).numpy()
    # activation INT8 (K7): one group of x all zero (scale 1 rule), one with a large outlier
    for tag, (o, i), g in (("sq", (256, 256), 128), ("g64", (96, 192), 64)):
        w, x = rnd(o, i), rnd(i, scale=1.0)
        x[:g] = 0.0
        x[g + 3] = 40.0
        blob = encode_scale_u8_grouped(w, group_size=g)
        y = lg.lut2_gemv(blob, x, out_features=o, in_features=i, activation_int8=True)
        out[f"i8_{tag}/blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"i8_{tag}/x"] = x.numpy()
        out[f"i8_{tag}/y"] = y.numpy()
        out[f"i8_{tag}/shape"] = np.array([o, i])
    # activation INT8 three maps (K14)
    os.environ["RWKV_LUT_ACTIVATION_INT8"] = "1"
    blobs = tuple(encode_scale_u8_grouped(rnd(C, 2 * C), group_size=128) for _ in range(3))
    xs = tuple(rnd(2 * C, scale=1.0) for _ in range(3))
    ys = lg.lut2_tmix_qkv_gemv_batched(blobs, xs, out_features=C, in_features=2 * C)
    os.environ["RWKV_LUT_ACTIVATION_INT8"] = "0"
    for j in range(3):
        out[f"i8_qkv/blob{j}"] = np.frombuffer(blobs[j], np.uint8).copy()
        out[f"i8_qkv/x{j}"] = xs[j].numpy()
    out["i8_qkv/y"] = torch.stack(list(ys)).numpy()
    np.savez_compressed(HERE / "gemv_extra.npz", **out)


class _StubProvider:
    """Duck-typed provider exposing the fused-blob protocol
    (``weight_provider.py:660-667``)."""

    def __init__(self, blobs, tmix):
        self._blobs = blobs
        self._tmix = tmix
        self._prepared_layers = {}

    def _use_fused_lut_matmul(self):
        return True

    def get_fused_lut_blob(self, name):
        return self._blobs.get(name)

    def get_fused_tmix_blobs(self, prefix):
        return self._tmix.get(prefix)


def forward_fixture(policy: str) -> None:
    sys.path.insert(0, str(REPO / "ssd-rwkv-engine_b200"))
    from rwkv_b200 import synth
    from rwkv_ssd.runtime.packed_block_forward import forward_block_packed
    from rwkv_ssd.runtime.pack_codec import decode_scale_u8_grouped_to_tensor, encode_scale_u8_grouped
    from rwkv_ssd.runtime.rwkv7_linear import matvec_z_or_lut
    from rwkv_ssd.runtime.trinity_codec import encode_trinity_lut2
    import torch.nn.functional as F

    os.environ["RWKV_LUT_KERNEL"] = "c" if policy == "sg8" else "auto"
    shape = synth.PRESETS["tiny"]
    C, H, N, L = shape.n_embd, shape.n_head, shape.head_size, shape.n_layer
    sd = synth.generate_state_dict(shape, SEED, "cpu")
    blobs: dict[str, tuple[bytes, int, int]] = {}
    z: dict[str, torch.Tensor] = {}
    hashes: dict[str, np.ndarray] = {}
    for name, t in sd.items():
        codec = synth.codec_for(name, tuple(t.shape), policy)
        if codec == "none":
            z[name] = t.reshape(-1).clone()
            continue
        if codec == "sg8":
            blob = encode_scale_u8_grouped(t, group_size=128)
        else:
            blob = encode_trinity_lut2(t, codebook="groupwise_kmeans_fp16", group_size=64)
        hashes[f"sha256/{name}"] = np.array(_sha(blob))
        blobs[name] = (blob, int(t.shape[0]), int(t.shape[1]))
    # skeleton tensors a provider would decode densely (r_k, emb)
    for i in range(L):
        nm = f"blocks.{i}.att.r_k"
        b = blobs.pop(nm)[0]
        z[nm] = decode_scale_u8_grouped_to_tensor(b, _entry(nm, (H, N), len(b), "scale_u8_grouped"),
                                                  torch.device("cpu")).reshape(-1)
    eb = blobs.pop("emb.weight")[0]
    emb = decode_scale_u8_grouped_to_tensor(eb, _entry("emb.weight", (shape.vocab, C), len(eb),
                                                       "scale_u8_grouped"), torch.device("cpu"))
    emb = F.layer_norm(emb, (C,), weight=z["blocks.0.ln0.weight"], bias=z["blocks.0.ln0.bias"])
    tmix = {}
    for i in range(L):
        p = f"blocks.{i}.att."
        tmix[p] = (tuple(blobs[p + s][0] for s in ("receptance.weight", "key.weight",
                                                    "value.weight", "output.weight")), C, C)
    prov = _StubProvider(blobs, tmix)

    state = []
    for _ in range(L):
        state += [torch.zeros(C), torch.zeros(H, N, N), torch.zeros(C)]

    def step(tok):
        x = emb[int(tok)].clone()
        v_first = torch.empty(0)
        for i in range(L):
            x, v_first, _ = forward_block_packed(i, x, state, v_first, z, prov, n_head=H, head_size=N,
                                                 n_embd=C, act_dtype=torch.float32)
        x = F.layer_norm(x, (C,), weight=z["ln_out.weight"], bias=z["ln_out.bias"])
        return matvec_z_or_lut(z, "head.weight", x, prov, act_dtype=torch.float32)

    prompt = synth.seeded_prompt(PROMPT_LEN, shape.vocab, SEED)
    rows, ids = [], []
    logits = None
    for t in prompt:
        logits = step(t)
        rows.append(logits.numpy().copy())
    for i in range(GEN_LEN):
        nxt = int(logits.argmax().item())
        ids.append(nxt)
        if i + 1 < GEN_LEN:
            logits = step(nxt)
            rows.append(logits.numpy().copy())
    out = {"prompt": np.array(prompt), "ids": np.array(ids), "logits": np.stack(rows),
           "seed": np.array(SEED), **hashes}
    for j, s in enumerate(state):
        out[f"state/{j}"] = s.numpy().astype(np.float32)
    np.savez_compressed(HERE / f"forward_tiny_{policy}.npz", **out)


def main() -> None:
    if not (REF_ROOT / "rwkv_ssd").is_dir():
        raise SystemExit(f"reference tree not found at {REF_ROOT}")
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    os.environ["RWKV_LUT_ACTIVATION_FP32"] = "1"
    os.environ.setdefault("OMP_NUM_THREADS", "8")
    torch.set_num_threads(1)
    tmp = _prepare_reference()
    try:
        which = set(sys.argv[1:]) or {"codec", "gemv", "extra", "forward"}
        if "codec" in which:
            codec_fixtures()
        if "gemv" in which:
            gemv_fixtures()
        if "extra" in which:
            extra_fixtures()
        if "forward" in which:
            forward_fixture("sg8")
            forward_fixture("lut2")
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
