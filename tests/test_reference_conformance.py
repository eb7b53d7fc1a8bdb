"""The drop-in boundary checked against the reference's own plugin API.

Runs only where the reference source tree is present (the development
container; ``RWKV_REF_ROOT`` overrides its location) and skips elsewhere.  The
reference package is copied to a temporary directory, its
``rwkv_ssd/backends/factory.py`` gets the ``cuda_b200`` lines that
INTEGRATION.md gives, and a child process (so no test shares the patched
modules) checks, with the reference's classes:

* ``create_backend("cuda_b200")`` returns a ``CudaB200Backend`` that is a
  reference ``PackBackend`` (``is_pack_backend``: the engine routes it through
  ``_generate_pack``) with no abstract method left unimplemented;
* every public method of ``PackBackend`` / ``RecurrentBackend`` exists on it
  with the reference's parameter names, kinds and optionality (extra
  parameters only with defaults);
* ``RecurrentState`` and the error types are the reference's own;
* ``supports_streaming_mode`` accepts the key, and ``ensure_v0_backend`` raises
  the reference's ``BackendNotAvailableError`` on a host without an sm_100a GPU;
* ``capabilities()["declared"]`` has every key the reference's probe reports.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
REF_ROOT = Path(os.environ.get("RWKV_REF_ROOT", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REF_ROOT / "rwkv_ssd" / "backends" / "factory.py").is_file(),
                                reason="reference source tree not present")

# The factory lines of INTEGRATION.md, inserted at the places it names.
_PATCHES = [
    ('OPTIONAL_BACKENDS = frozenset({"rwkvcpp", "cpp"})\n',
     'OPTIONAL_BACKENDS = frozenset({"rwkvcpp", "cpp"})\n'
     'CUDA_B200_BACKENDS = frozenset({"cuda_b200", "b200"})\n'),
    ('    if key in ("albatross", "alb"):\n        return AlbatrossBackend()\n',
     '    if key in ("albatross", "alb"):\n        return AlbatrossBackend()\n'
     '    if key in CUDA_B200_BACKENDS:\n'
     '        from rwkv_b200.backend import CudaB200Backend  # lazy: torch + CUDA only when selected\n'
     '        return CudaB200Backend()\n'),
    ('    return key in (*SUPPORTED_BACKENDS, *ALBATROSS_BACKENDS)\n',
     '    return key in (*SUPPORTED_BACKENDS, *ALBATROSS_BACKENDS, *CUDA_B200_BACKENDS)\n'),
    ('    if key in SUPPORTED_BACKENDS:\n        return\n',
     '    if key in SUPPORTED_BACKENDS:\n        return\n'
     '    if key in CUDA_B200_BACKENDS:\n'
     '        from rwkv_b200.backend import ensure_v0_backend as _b200_gate\n'
     '        _b200_gate(key)\n'
     '        return\n'),
]

_CHECK = textwrap.dedent('''
    import inspect
    import torch
    from rwkv_ssd.backends import factory
    from rwkv_ssd.backends.base import RecurrentBackend
    from rwkv_ssd.backends.capabilities import probe_backend_capabilities
    from rwkv_ssd.backends.pack_backend import PackBackend
    from rwkv_ssd.backends.synthetic import SyntheticBackend
    from rwkv_ssd.runtime import errors
    from rwkv_ssd.runtime.generation_control import GenerationCancelled
    from rwkv_ssd.runtime.state_cache import RecurrentState

    b = factory.create_backend("cuda_b200")
    from rwkv_b200 import backend as mod
    assert mod.REFERENCE_TYPES
    assert isinstance(b, mod.CudaB200Backend)
    assert isinstance(b, PackBackend) and factory.is_pack_backend(b)
    assert not getattr(mod.CudaB200Backend, "__abstractmethods__", set()), mod.CudaB200Backend.__abstractmethods__
    assert mod.RecurrentState is RecurrentState
    assert mod.BackendNotAvailableError is errors.BackendNotAvailableError
    assert mod.CapabilityNotSupportedError is errors.CapabilityNotSupportedError
    assert mod.GenerationCancelled is GenerationCancelled
    assert factory.supports_streaming_mode("cuda_b200") and factory.supports_streaming_mode("b200")

    def check(ref_cls):
        n = 0
        for name, ref in vars(ref_cls).items():
            if name.startswith("_"):
                continue
            ours = inspect.getattr_static(mod.CudaB200Backend, name)
            if isinstance(ref, property):
                assert isinstance(ours, property), name
                n += 1
                continue
            if not callable(ref):
                continue
            assert callable(ours), name
            rp = inspect.signature(ref).parameters
            op = inspect.signature(ours).parameters
            for pname, p in rp.items():
                assert pname in op, (name, pname)
                q = op[pname]
                assert q.kind == p.kind, (name, pname, q.kind, p.kind)
                if p.default is not inspect.Parameter.empty:
                    assert q.default is not inspect.Parameter.empty, (name, pname)
            for pname, q in op.items():
                if pname not in rp:
                    assert q.default is not inspect.Parameter.empty or q.kind in (q.VAR_POSITIONAL, q.VAR_KEYWORD), \\
                        (name, pname)
            n += 1
        return n

    n = check(PackBackend) + check(RecurrentBackend)
    assert n >= 20, n

    if not torch.cuda.is_available():
        try:
            factory.ensure_v0_backend("cuda_b200")
        except errors.BackendNotAvailableError:
            pass
        else:
            raise AssertionError("ensure_v0_backend accepted a host without a B200")

    ref_keys = set(probe_backend_capabilities(SyntheticBackend())["declared"])
    ours = b.capabilities()["declared"]
    assert ref_keys <= set(ours), sorted(ref_keys - set(ours))
    assert ours["pack_streaming"] in (True, False)
    print("conformance ok", n)
''')


def test_backend_conforms_to_reference_plugin_api(tmp_path):
    dst = tmp_path / "rwkv_ssd"
    shutil.copytree(REF_ROOT / "rwkv_ssd", dst, ignore=shutil.ignore_patterns("*.dll", "__pycache__", "*.so"))
    fac = dst / "backends" / "factory.py"
    src = fac.read_text()
    for old, new in _PATCHES:
        assert old in src, old
        src = src.replace(old, new, 1)
    fac.write_text(src)
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(tmp_path), str(REPO / "ssd-rwkv-engine_b200"), str(REPO)])
    env["CUDA_VISIBLE_DEVICES"] = env.get("CUDA_VISIBLE_DEVICES", "")
    r = subprocess.run([sys.executable, "-c", _CHECK], env=env, cwd=str(tmp_path), capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "conformance ok" in r.stdout
