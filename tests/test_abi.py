"""The C ABI: libonnxsharp_cuda loads, exports every symbol that
include/*.h declares, and reports errors through status codes and
osc_last_error() without touching a device (host-side fault injection)."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import sys

import pytest

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))
DECL = re.compile(r"OSC_API\s+[\w\s\*]+?\b(osc_\w+)\s*\(")


def declared_symbols() -> list[str]:
    names = []
    for h in HEADERS:
        names += DECL.findall(h.read_text())
    return sorted(set(names))


def test_headers_declare_symbols():
    assert "osc_gemm_bias_f32" in declared_symbols()


def test_library_exports_every_declared_symbol():
    from onnxsharp_b200 import _lib

    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_table_covers_header():
    from onnxsharp_b200 import _lib

    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_version_and_empty_error():
    from onnxsharp_b200 import _lib

    assert _lib.load().osc_version() >= 100
    assert isinstance(_lib.last_error(), str)


def _run(code: str, env_extra: dict[str, str]) -> str:
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=ROOT, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout.strip()


CREATE = (
    "import ctypes as C; from onnxsharp_b200 import _lib; l=_lib.load(); h=C.c_void_p();"
    "st=l.osc_create(0, C.byref(h)); print(st, _lib.last_error())"
)


def test_fault_injection_on_create_touches_no_device():
    out = _run(CREATE, {"OSC_FAULT": "create"})
    st, msg = out.split(" ", 1)
    assert int(st) == 6 and "injected" in msg  # OSC_EFAULT_INJECTED


def test_create_without_gpu_reports_error_not_crash():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    out = _run(CREATE, {"OSC_FAULT": ""})
    st, _ = out.split(" ", 1)
    assert int(st) in (3, 1)  # OSC_ECUDA (no driver) or OSC_EINVAL (no device)


def test_null_arguments_are_rejected():
    from onnxsharp_b200 import _lib

    lib = _lib.load()
    assert lib.osc_create(0, None) == 1  # OSC_EINVAL
    assert lib.osc_synchronize(None, 10) == 1
    assert lib.osc_gemm_bias_f32(None, None, 1, 1, 0, None, None, 0, None, 0) == 1
    assert lib.osc_destroy(None) == 0
