"""CPU checks of the C ABI boundary (no GPU needed): the sm_100a library and
the C++ host layer load, and export every entry point their headers declare."""
import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "pixal3d" / "cpp_b200"


def declared(header: Path) -> list[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(p3d_[a-z0-9_]+)\s*\(", text)))


def test_kernel_library_exports_every_declared_symbol():
    lib_path = PKG / "libp3dcuda.so"
    if not lib_path.exists():
        pytest.skip("libp3dcuda.so not built (run python -m pixal3d.cpp_b200.build)")
    lib = ctypes.CDLL(str(lib_path))
    names = declared(REPO / "include" / "p3d.h")
    assert len(names) > 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_loads_and_reports_version():
    from pixal3d.cpp_b200 import _lib
    assert _lib.lib.p3d_version() >= 1
    assert _lib.lib.p3d_coord_hash_capacity(1000) == 2048
    assert _lib.lib.p3d_neighbor_map27_workspace(1000) >= 2048 * 12


def test_context_creation_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from pixal3d.cpp_b200 import _lib
    h = ctypes.c_void_p()
    rc = _lib.lib.p3d_ctx_create(0, None, ctypes.byref(h))
    assert rc == _lib.P3D_ERR_NO_DEVICE
