"""GGUF pack loading through the reference API on the CPU (no device work):
SLatFlowModel::load(path, component, load_tensors=false) of packs written by
tests/gguf_pack.py, and the refusals the reference's loader makes
(src/pack.cpp:127-260, src/slat_flow.cpp:1239-1281): unknown component,
component absent from the pack, bad magic, foreign architecture, truncated
header, missing hyperparameter, tensor data beyond the end of the file.
The device-side load + forward is in tests/test_gpu_host_api.py."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests import gguf_pack as G
from tests._models import random_flow_weights

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "pixal3d" / "cpp_b200"
HP = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2, num_heads=2)


@pytest.fixture(scope="module")
def tool(tmp_path_factory):
    if not (PKG / "libpixal3d_b200.so").exists():
        pytest.skip("host library not built")
    d = tmp_path_factory.mktemp("gguf")
    exe = d / "gguf_info"
    subprocess.run(["g++", "-O1", "-std=c++17", f"-I{PKG / 'host' / 'include'}", str(REPO / "tests" / "cpp" / "gguf_info.cpp"),
                    f"-L{PKG}", "-lpixal3d_b200", "-lp3dcuda", f"-Wl,-rpath,{PKG}", "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    return exe, d


def _pack(path, meta_edit=None):
    w = random_flow_weights(np.random.default_rng(5), HP)
    meta = G.flow_metadata("shape_flow_512", HP)
    if meta_edit:
        meta_edit(meta)
    G.write_pack(path, meta, G.flow_tensors("sh512", w))


def _run(tool, path, component="shape_flow_512"):
    exe, _ = tool
    r = subprocess.run([str(exe), str(path), component], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    return r.stdout.strip()


def test_header_load(tool):
    p = tool[1] / "ok.gguf"
    _pack(p)
    assert _run(tool, p) == f"ok {10 + 21 * HP.num_blocks} 128 2 2 0"


def test_refusals(tool):
    d = tool[1]
    p = d / "ok.gguf"
    _pack(p)
    assert _run(tool, p, "texture_flow_1024").startswith("error GGUF pack does not contain SLat flow component")
    assert _run(tool, p, "flow_9000").startswith("error unsupported SLat flow component")
    bad = d / "magic.gguf"
    bad.write_bytes(b"GGML" + p.read_bytes()[4:])
    assert _run(tool, bad).startswith("error not a GGUF file")
    arch = d / "arch.gguf"
    _pack(arch, lambda m: m.update({"general.architecture": "llama"}))
    assert _run(tool, arch) == "error unexpected GGUF architecture: llama"
    miss = d / "miss.gguf"
    _pack(miss, lambda m: m.pop("pixal3d.shape_flow_512.num_heads"))
    assert _run(tool, miss) == "error missing GGUF metadata: pixal3d.shape_flow_512.num_heads"
    share = d / "share.gguf"
    _pack(share, lambda m: m.update({"pixal3d.shape_flow_512.share_mod": False}))
    assert _run(tool, share) == "error SLat flow currently requires pe_mode=rope and share_mod=true"
    raw = p.read_bytes()
    trunc = d / "trunc.gguf"
    trunc.write_bytes(raw[:200])
    assert _run(tool, trunc).startswith("error truncated GGUF")
    short = d / "short.gguf"
    short.write_bytes(raw[:len(raw) - 4096])
    assert _run(tool, short).startswith("error GGUF tensor payload is outside the file")


def test_writer_stores_expected_values():
    a = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0], np.float32)
    np.testing.assert_array_equal(G.stored(a, G.GGML_F16), a.astype(np.float16).astype(np.float32))
    b = G.stored(a, G.GGML_BF16)
    assert np.all(np.abs(b - a) <= np.abs(a) * 2 ** -8)
    np.testing.assert_array_equal(G.stored(b, G.GGML_BF16), b)
