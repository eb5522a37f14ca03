"""Regenerate the golden vectors under tests/golden/ from the reference itself.

Run where the reference checkout is mounted (it is not on the GPU box):

    python tests/golden/make_golden.py [--ref /root/reference]

1. Builds the reference CPU path and its deterministic numeric fixtures with
   oracle/Makefile (sources compiled where they lie; outputs in oracle/_ref/).
2. Runs each fixture and stores its stdout verbatim as <fixture>.txt.  These
   are the reference's own known-answer outputs (max_digits10 floats).
3. Calls the compiled reference through oracle/reflib.py on small seeded
   inputs and stores inputs + outputs in ref_vectors.npz.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

FIXTURES = [
    ("sparse_numeric_fixture", []),
    ("sparse_transformer_numeric_fixture", []),
    ("flow_sampler_numeric_fixture", []),
    ("slat_flow_numeric_fixture", []),
    ("slat_decoder_numeric_fixture", ["--upsample"]),
    ("flow_numeric_fixture", []),
]


def build(ref: str) -> None:
    subprocess.run(["make", "-C", str(REPO / "oracle"), f"REF={ref}", "-j8"], check=True)


def run_fixtures() -> None:
    for name, args in FIXTURES:
        exe = REPO / "oracle" / "_ref" / "bin" / name
        out = subprocess.run([str(exe), *args], check=True, capture_output=True, text=True).stdout
        (HERE / f"{name}.txt").write_text(out)
        print("wrote", name, len(out), "bytes")


def ref_vectors() -> None:
    from oracle import reflib
    from pixal3d.cpp_b200.workloads import shell_coords, batched

    reflib.set_threads(8)
    rng = np.random.default_rng(1234)
    v = {}
    # Small shell, two batch items (second one shifted so the sets differ).
    c0 = shell_coords(16, 5.0, 1.0)
    c1 = shell_coords(16, 6.0, 0.8)
    c1[:, 0] = 1
    coords = np.ascontiguousarray(np.concatenate([c0, c1]))
    n = coords.shape[0]
    v["coords"] = coords
    v["nbr"] = reflib.neighbor_map27(coords, 2, (16, 16, 16))
    v["fingerprint"] = np.array([reflib.coords_fingerprint(coords)], dtype=np.uint64)
    x = rng.standard_normal((n, 8)).astype(np.float32)
    w = (rng.standard_normal((27, 12, 8)) / np.sqrt(27 * 8)).astype(np.float32)
    b = (rng.standard_normal(12) * 0.1).astype(np.float32)
    v["conv_x"], v["conv_w"], v["conv_b"] = x, w, b
    v["conv_out"] = reflib.subm_conv3d(coords, x, w, b, 2, (16, 16, 16))
    dc, df, dshape = reflib.downsample_mean(coords, x, 2, 2, (16, 16, 16))
    v["down_coords"], v["down_feats"] = dc, df
    xs = rng.standard_normal((n, 8 * 3)).astype(np.float32)
    sd = rng.standard_normal((n, 8)).astype(np.float32)
    v["c2s_x"], v["c2s_mask"] = xs, sd
    cc, cf = reflib.channel_to_spatial(coords, xs, 2, sd, 2, (16, 16, 16))
    v["c2s_coords"], v["c2s_feats"] = cc, cf
    q = rng.standard_normal((n, 16)).astype(np.float32)
    k = rng.standard_normal((n, 16)).astype(np.float32)
    vv = rng.standard_normal((n, 16)).astype(np.float32)
    v["attn_q"], v["attn_k"], v["attn_v"] = q, k, vv
    v["attn_out"] = reflib.sdpa(coords, q, k, vv, 2, 8, 0.35, 2, (16, 16, 16))
    v["rope_out"] = reflib.rope(coords, q, 2, 8, 1.0, 10000.0, 2, (16, 16, 16))
    g = (np.abs(rng.standard_normal(16)) + 0.5).astype(np.float32)
    v["rms_gamma"] = g
    v["rms_out"] = reflib.rms_norm(coords, q, 2, 8, g, 2, (16, 16, 16))
    np.savez_compressed(HERE / "ref_vectors.npz", **v)
    print("wrote ref_vectors.npz", n, "points")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("P3D_REFERENCE", "/root/reference"))
    a = ap.parse_args()
    build(a.ref)
    run_fixtures()
    ref_vectors()


if __name__ == "__main__":
    main()
