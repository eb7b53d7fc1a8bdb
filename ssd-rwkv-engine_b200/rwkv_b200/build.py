"""Build the sm_100a shared library ``_lib/librwkvb200.so`` with nvcc.

The library is built in-tree so it travels with the source checkout; there is
no JIT cache.  ``python -m rwkv_b200.build`` (with ``ssd-rwkv-engine_b200`` on
``sys.path``) or ``rwkv_b200.build.build()`` compiles every ``csrc/*.cu`` for
``compute_100a`` / ``sm_100a`` only.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # ssd-rwkv-engine_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"      # repository include/ (the C ABI header)
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "librwkvb200.so"
STAMP = LIB_DIR / "librwkvb200.stamp"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
              "-Xptxas", "-O3", "-cudart", "static"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).is_file():
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC)")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile the library unless an up-to-date build exists."""
    digest = _digest()
    if not force and LIB.is_file() and STAMP.is_file() and STAMP.read_text().strip() == digest:
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    procs = []
    for src in _sources():
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if out and (verbose or ptxas_info or p.returncode):
            print(out, file=sys.stderr)
        if p.returncode:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    STAMP.write_text(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv))
