"""The C-ABI library loads and exports every symbol include/*.h declares;
argument validation happens on the host before any device call (CPU only).
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(dfl_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared_functions()
    assert "dfl_verify_qmm_w4g64" in names
    assert len(names) >= 5


def test_library_exports_every_declared_symbol(pkg):
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the binding, and vice versa
    assert sorted(_lib.SIGNATURES) == _declared_functions()


def test_status_strings_and_version(pkg):
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    assert b"sm_100a" in lib.dfl_version()
    assert lib.dfl_status_string(0) == b"ok"
    assert lib.dfl_status_string(2) == b"unsupported shape"


@pytest.mark.parametrize("m,k,n", [(0, 64, 8), (33, 64, 8), (16, 96, 8), (16, 0, 8), (16, 64, 0)])
def test_qmm_rejects_bad_shapes_before_touching_the_device(pkg, m, k, n):
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    fake = ctypes.c_void_p(256)
    st = lib.dfl_verify_qmm_w4g64(fake, fake, fake, fake, fake, fake, 1 << 20, m, k, n, None)
    assert st == 2
    status = ctypes.c_int(-1)
    assert lib.dfl_verify_qmm_workspace_bytes(m, k, n, ctypes.byref(status)) == 0
    assert status.value == 2


def test_qmm_rejects_null_pointers(pkg):
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    fake = ctypes.c_void_p(256)
    st = lib.dfl_verify_qmm_w4g64(None, fake, fake, fake, fake, fake, 1 << 20, 16, 64, 8, None)
    assert st == 1


def test_qmm_rejects_misaligned_activations(pkg):
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    fake = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(258)
    st = lib.dfl_verify_qmm_w4g64(odd, fake, fake, fake, fake, fake, 1 << 20, 16, 64, 8, None)
    assert st == 3


def test_python_surface_refuses_cpu_tensors(pkg):
    import torch

    x = torch.zeros(16, 64, dtype=torch.bfloat16)
    w = torch.zeros(8, 8, dtype=torch.int32)
    s = torch.zeros(8, 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.verify_matmul(x, w, s, s)
    with pytest.raises(NotImplementedError):
        pkg.verify_matmul(x, w, s, s, bits=8)
