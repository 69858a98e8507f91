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


def _declarations():
    """(return type, name, [parameter types]) of every declaration in include/*.h."""
    out = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for ret, name, params in re.findall(
                r"([A-Za-z_][A-Za-z0-9_ \*]*?)\b(dfl_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
            ps = [] if params.strip() in ("", "void") else [p.strip() for p in params.split(",")]
            types = [p.rsplit(" ", 1)[0] if not p.endswith("*") else p for p in ps]
            out.append((ret.strip(), name, types))
    return out


def _ctypes_kind(t):
    if t in (ctypes.c_void_p, ctypes.c_char_p) or isinstance(t, type(ctypes.POINTER(ctypes.c_int))):
        return "pointer"
    # c_size_t and c_uint64 are the same ctypes class on LP64 Linux
    return {ctypes.c_int: "int", ctypes.c_size_t: "u64", ctypes.c_uint64: "u64",
            ctypes.c_float: "float"}.get(t, repr(t))


def _c_kind(t):
    t = t.replace("const ", "").strip()
    if t.endswith("*"):
        return "pointer"
    return {"int": "int", "int32_t": "int", "size_t": "u64", "uint64_t": "u64",
            "float": "float"}.get(t, t)


def test_binding_signatures_match_the_header(pkg):
    """Every ctypes signature has the header's arity and, position by position,
    the same kind of argument (pointer / 32-bit int / 64-bit size), so no call passes a
    64-bit pointer where the library reads a 32-bit int or the reverse."""
    from dflash_mlx_b200 import _lib

    decls = _declarations()
    assert sorted(n for _, n, _ in decls) == _declared_functions()
    for ret, name, params in decls:
        restype, argtypes = _lib.SIGNATURES[name]
        assert [_ctypes_kind(a) for a in argtypes] == [_c_kind(p) for p in params], name
        assert _ctypes_kind(restype) == _c_kind(ret), name
