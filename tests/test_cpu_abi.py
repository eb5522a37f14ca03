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


REFERENCE_API = [
    "pixal3d::SparseTensorF32::valid", "pixal3d::VarLenTensorF32::valid", "pixal3d::sparse_linear",
    "pixal3d::varlen_linear", "pixal3d::sparse_layer_norm", "pixal3d::sparse_downsample_mean",
    "pixal3d::sparse_channel_to_spatial", "pixal3d::sparse_scaled_dot_product_attention",
    "pixal3d::sparse_cross_attention", "pixal3d::sparse_rotary_position_embedding",
    "pixal3d::sparse_multihead_rms_norm", "pixal3d::varlen_multihead_rms_norm",
    "pixal3d::sparse_submanifold_conv3d", "pixal3d::sparse_transformer_cross_block_f32",
    "pixal3d::flow_euler_sample_f32", "pixal3d::slat_flow_forward_f32", "pixal3d::SLatFlowModel::forward",
    "pixal3d::SLatFlowModel::sample", "pixal3d::SLatFlowModel::load", "pixal3d::SLatFlowModel::bind",
    "pixal3d::sparse_convnext_block_f32", "pixal3d::sparse_resblock_c2s_f32", "pixal3d::slat_decoder_forward_f32",
    "pixal3d::slat_decoder_upsample_coords_f32", "pixal3d::SLatDecoderModel::decode",
    "pixal3d::SLatDecoderModel::upsample_coords", "pixal3d::SLatDecoderModel::bind",
]


def test_host_library_exports_the_reference_api():
    """libpixal3d_b200.so defines the reference's include/pixal3d functions
    (C++ names, same signatures), so a reference caller links against it."""
    import subprocess
    lib_path = PKG / "libpixal3d_b200.so"
    if not lib_path.exists():
        pytest.skip("libpixal3d_b200.so not built")
    out = subprocess.run(["nm", "-DC", "--defined-only", str(lib_path)], capture_output=True, text=True).stdout
    missing = [f for f in REFERENCE_API if f + "(" not in out]
    assert not missing, missing


def test_host_api_fails_cleanly_without_gpu(tmp_path):
    """Without a B200 every host-API call returns false with a message (no CPU fallback)."""
    import subprocess
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    src = tmp_path / "t.cpp"
    src.write_text(r'''
#include "pixal3d/sparse.h"
#include <cstdio>
int main() {
    pixal3d::SparseTensorF32 x; x.batch_size = 1; x.channels = 1; x.spatial_x = x.spatial_y = x.spatial_z = 2;
    x.coords = {0, 0, 0, 0}; x.feats = {1.0f};
    std::string e; float w = 2.0f;
    pixal3d::SparseTensorF32 y;
    const bool ok = pixal3d::sparse_linear(x, &w, nullptr, 1, y, &e);
    std::printf("%d %s\n", ok ? 1 : 0, e.c_str());
    return ok ? 1 : 0;
}
''')
    exe = tmp_path / "t"
    r = subprocess.run(["g++", "-std=c++17", f"-I{PKG / 'host' / 'include'}", str(src), f"-L{PKG}", "-lpixal3d_b200",
                        "-lp3dcuda", f"-Wl,-rpath,{PKG}", "-o", str(exe)], capture_output=True, text=True)
    if r.returncode != 0 or not (PKG / "libpixal3d_b200.so").exists():
        pytest.skip("host library not built: " + r.stderr[-200:])
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.startswith("0 ") and "device" in r.stdout, r.stdout + r.stderr
