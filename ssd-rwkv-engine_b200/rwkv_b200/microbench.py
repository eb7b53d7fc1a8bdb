"""Kernel microbenchmark of the packed products and the WKV7 update.

``python -m rwkv_b200.microbench`` (with ``ssd-rwkv-engine_b200`` on
``sys.path``) prints one JSON line per case:

* packed product ``y = x @ W^T`` for N x K in {2560x2560, 10240x2560,
  2560x10240, 16384x4096, 65536x4096 (head)} at batch B in {1, 8, 64, 256} for
  the SG8 g128 and LUT2 ``TR2\\x04`` g64 codecs.  B = 1 is the GEMV
  (``rwkvb_gemv_f32``); SG8 at 1 < B <= 64 is the tcgen05 batched product
  (``rwkvb_gemm_sg8_f32``); B = 256 runs it over four 64-row slices; LUT2 at
  B > 1 runs one GEMV per row (there is no batched LUT2 product yet).
* WKV7 state update (``rwkvb_wkv7_f32``) at B in {1, 64} sessions x 64 heads x
  64 x 64 fp32 state, inputs ~ N(0, 1), decay ``exp(-0.606531 sigmoid(w))``
  (the model's) and ``exp(-exp(w))``.

Inputs are seeded synthetic (codes from the reference codecs applied to
N(0, 0.02) weights; x ~ N(0, 1)); every timed call is preceded by a write of a
buffer larger than L2 when the working set fits in L2.  Times are CUDA events
on the launching stream; ``frac`` is against the measured HBM copy bandwidth
(``MEASURED_PEAKS.json``) or the 6650 GB/s fallback.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
from pathlib import Path

import torch

from . import lut_gemm_fused as lg
from . import native, synth
from .residency import WeightArena

SHAPES = [(2560, 2560), (10240, 2560), (2560, 10240), (16384, 4096), (65536, 4096)]
BATCHES = [1, 8, 64, 256]


def _peak() -> tuple[float, str]:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class _Timer:
    def __init__(self, iters: int, flush: torch.Tensor | None):
        self.iters, self.flush = iters, flush

    def __call__(self, fn) -> float:
        """Average ms per call of ``fn`` (device time, CUDA events)."""
        for _ in range(2):
            fn()
        total = 0.0
        for _ in range(self.iters):
            if self.flush is not None:
                self.flush.add_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        return total / self.iters


def _packed(rows: int, cols: int, codec: str, seed: int):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn((rows, cols), generator=gen, device="cuda") * 0.02
    blob = synth.encode_sg8(w, 128) if codec == "sg8" else synth.encode_lut2(w, 64)
    del w
    arena = WeightArena([("w", blob, (rows, cols), codec)], torch.device("cuda", torch.cuda.current_device()))
    return arena, int(blob.numel())


def product_cases(timer: _Timer, peak: float, shapes, batches, codecs) -> list[dict]:
    lib = native.lib()
    out = []
    stream = torch.cuda.current_stream().cuda_stream
    for codec in codecs:
        for (n, k) in shapes:
            arena, wbytes = _packed(n, k, codec, n + k)
            desc = arena["w"].desc
            for b in batches:
                x = torch.randn((b, k), device="cuda")
                y = torch.empty((b, n), device="cuda")
                if b == 1:
                    def fn():
                        native.check(lib.rwkvb_gemv_f32(y.data_ptr(), ctypes.byref(desc), x.data_ptr(), stream),
                                     "rwkvb_gemv_f32")
                    how = "rwkvb_gemv_f32"
                elif codec == "sg8":
                    def fn():
                        for r0 in range(0, b, 64):
                            nb = min(64, b - r0)
                            native.check(lib.rwkvb_gemm_sg8_f32(y[r0].data_ptr(), ctypes.byref(desc),
                                                                x[r0].data_ptr(), nb, None, stream),
                                         "rwkvb_gemm_sg8_f32")
                    how = "rwkvb_gemm_sg8_f32" + (f" x{(b + 63) // 64}" if b > 64 else "")
                else:
                    def fn():
                        for r in range(b):
                            native.check(lib.rwkvb_gemv_f32(y[r].data_ptr(), ctypes.byref(desc), x[r].data_ptr(),
                                                            stream), "rwkvb_gemv_f32")
                    how = f"rwkvb_gemv_f32 x{b}"
                ms = timer(fn)
                passes = 1 if (b == 1 or codec == "sg8" and b <= 64) else ((b + 63) // 64 if codec == "sg8" else b)
                alg = wbytes * passes + 4 * b * (k + n)
                gbs = alg / (ms * 1e-3) / 1e9
                out.append({"case": "packed_product", "codec": codec, "N": n, "K": k, "batch": b, "entry": how,
                            "ms": ms, "weight_bytes": wbytes, "algorithmic_bytes": alg, "GB/s": gbs,
                            "frac": gbs / peak, "TFLOP/s": 2.0 * n * k * b / (ms * 1e-3) / 1e12})
            del arena
            torch.cuda.empty_cache()
    return out


def wkv_cases(timer: _Timer, peak: float, batches=(1, 64)) -> list[dict]:
    out = []
    H, N = 64, 64
    for b in batches:
        for mode in (0, 1):
            gen = torch.Generator(device="cuda").manual_seed(7 + b)
            state = torch.randn((b, H, N, N), generator=gen, device="cuda") * 0.1
            vec = [torch.randn((b, H * N), generator=gen, device="cuda") for _ in range(6)]
            kk = torch.nn.functional.normalize(vec[4].view(b, H, N), dim=-1).reshape(b, H * N)
            a = torch.sigmoid(vec[5])

            def fn():
                lg.wkv7(state, vec[0], vec[1], vec[2], vec[3], kk, a, decay_mode=mode)
            ms = timer(fn)
            alg = 2 * state.numel() * 4 + 7 * b * H * N * 4
            gbs = alg / (ms * 1e-3) / 1e9
            out.append({"case": "wkv7", "batch": b, "heads": H, "decay": "exp(-0.606531*sigmoid(w))" if mode == 0
                        else "exp(-exp(w))", "ms": ms, "algorithmic_bytes": alg, "GB/s": gbs, "frac": gbs / peak})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--quick", action="store_true", help="two shapes, batches 1 and 64")
    args = ap.parse_args()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    peak, kind = _peak()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB > L2
    timer = _Timer(args.iters, flush)
    shapes = SHAPES[:2] if args.quick else SHAPES
    batches = [1, 64] if args.quick else BATCHES
    for rec in product_cases(timer, peak, shapes, batches, ("sg8", "lut2")) + wkv_cases(timer, peak):
        rec["peak_GB/s"] = peak
        rec["peak_kind"] = kind
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
