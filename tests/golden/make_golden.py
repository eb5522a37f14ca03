"""Regenerate the golden vectors under tests/golden/ from the reference itself.

Run where the reference checkout is mounted (it is not on the GPU box):

    python tests/golden/make_golden.py --ref <Pixal3D.cpp checkout>   (or $P3D_REFERENCE)

1. Builds the reference CPU path and its deterministic numeric fixtures with
   oracle/Makefile (sources compiled where they lie; outputs in oracle/_ref/).
2. Runs each fixture and stores its stdout verbatim as <fixture>.txt.  These
   are the reference's own known-answer outputs (max_digits10 floats).
3. Calls the compiled reference through oracle/reflib.py on small seeded
   inputs and stores inputs + outputs in ref_vectors.npz (sparse path) and
   projection_vectors.npz (projection conditioning).

    python tests/golden/make_golden.py --only configs

4. Runs the numpy oracle (oracle/oracle.py, pinned to the reference by
   tests/test_oracle_pin.py) on the BASELINE configurations at full size
   (tests/_configs.py: config-1 block at N=21,766, one config-2 forward at
   N=2 x 21,766 with 24 blocks) and stores the outputs with fingerprints of
   the seeded inputs in cfg1_block.npz and cfg2_forward.npz.  Needs no
   reference checkout; takes a few minutes of CPU.
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
    ("projection_numeric_fixture", []),
]


def build(ref: str) -> None:
    subprocess.run(["make", "-C", str(REPO / "oracle"), f"REF={ref}", "-j8"], check=True)


def run_fixtures() -> None:
    for name, args in FIXTURES:
        exe = REPO / "oracle" / "_ref" / "bin" / name
        out = subprocess.run([str(exe), *args], check=True, capture_output=True, text=True).stdout
        (HERE / f"{name}.txt").write_text(out)
        print("wrote", name, len(out), "bytes")
    # tests/cpp/projection_check.cpp built against the reference (oracle/Makefile)
    exe = REPO / "oracle" / "_ref" / "bin" / "projection_check_ref"
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    (HERE / "projection_check_reference.txt").write_text(out)
    print("wrote projection_check_reference", len(out), "bytes")


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


def _rot(ax: float, ay: float, az: float) -> np.ndarray:
    cx, sx, cy, sy, cz, sz = np.cos(ax), np.sin(ax), np.cos(ay), np.sin(ay), np.cos(az), np.sin(az)
    rx = np.array([[1, 0, 0], [0, cx, -sx], [0, sx, cx]])
    ry = np.array([[cy, 0, sy], [0, 1, 0], [-sy, 0, cy]])
    rz = np.array([[cz, -sz, 0], [sz, cz, 0], [0, 0, 1]])
    return rz @ ry @ rx


def _c2w(ax, ay, az, t) -> np.ndarray:
    m = np.eye(4)
    m[:3, :3] = _rot(ax, ay, az)
    m[:3, 3] = t
    return m.astype(np.float32).reshape(16)


def projection_vectors() -> None:
    """Projection conditioning (src/projection.cpp) on seeded inputs: a
    37x37 DINO-sized map sampled at a subset of the 64^3 shell from the front
    camera and from a rotated / translated camera (part of the shell falls
    outside the image or behind the camera), a dense two-view average, and
    relative camera matrices."""
    from oracle import reflib
    from oracle.oracle import ProjCamera
    from pixal3d.cpp_b200.workloads import shell_coords

    rng = np.random.default_rng(77)
    v = {}
    coords = np.ascontiguousarray(shell_coords()[::8])
    coords[:, 0] = 0
    fmap = rng.standard_normal((37, 37, 8)).astype(np.float32)
    v["coords"], v["fmap"] = coords, fmap
    front = ProjCamera(0.6, 2.0, 1.0)
    v["front_feats"], v["front_valid"] = reflib.project_at_coords(fmap, 64, 518, front, coords)
    # front view from distance 0.3 (inside the shell's extent), turned and
    # shifted: part of the shell is behind the camera or outside the image
    m = (_c2w(0.2, 0.0, 0.3, [0.05, 0.0, -0.1]).reshape(4, 4).astype(np.float64) @
         np.array([[1, 0, 0, 0], [0, 0, -1, -0.3], [0, 1, 0, 0], [0, 0, 0, 1]])).astype(np.float32).reshape(16)
    v["moved_c2w"] = m
    moved = ProjCamera(0.9, 2.0, 0.8, m)
    v["moved_feats"], v["moved_valid"] = reflib.project_at_coords(fmap, 64, 518, moved, coords)
    a = rng.standard_normal((9, 7, 5)).astype(np.float32)
    b = rng.standard_normal((9, 7, 5)).astype(np.float32)
    v["avg_map_a"], v["avg_map_b"] = a, b
    m2 = _c2w(0.0, 0.4, 0.0, [0.2, -2.2, 0.1])
    v["avg_c2w"] = m2
    v["avg_feats"], v["avg_valid"] = reflib.project_average([a, b], 8, 64, [ProjCamera(0.7, 2.2, 1.0),
                                                                        ProjCamera(0.7, 2.2, 1.0, m2)])
    c2w = np.stack([_c2w(0.1, 0.2, 0.3, [0.0, -2.0, 0.3]), _c2w(-0.4, 0.9, 0.1, [1.0, -1.5, 0.2]),
                    _c2w(0.7, -0.3, -1.1, [-0.5, 0.5, -2.0])])
    d = np.array([2.0, 1.7, 2.4], np.float32)
    v["rel_c2w"], v["rel_dist"] = c2w, d
    v["rel_out"] = reflib.relative_matrices(c2w, d)
    np.savez_compressed(HERE / "projection_vectors.npz", **v)
    print("wrote projection_vectors.npz", coords.shape[0], "points")


def config_goldens() -> None:
    import time

    from oracle import oracle as O
    from tests import _configs as K
    for name, make in (("cfg1_block", K.cfg1), ("cfg2_forward", K.cfg2)):
        coords, x, ts, offs, ctx, hp, w = make()
        t0 = time.perf_counter()
        out = O.slat_flow_forward(coords, x, ts, offs, ctx, None, hp, w)
        dt = time.perf_counter() - t0
        np.savez_compressed(HERE / f"{name}.npz", out=out.astype(np.float32),
                            inputs_fp=K.fingerprint(coords, x, ts, ctx), weights_fp=K.weights_fingerprint(w),
                            oracle_seconds=np.float64(dt))
        print(f"wrote {name}.npz: out {out.shape}, oracle {dt:.1f} s")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("P3D_REFERENCE"),
                    help="Pixal3D.cpp checkout (default $P3D_REFERENCE)")
    ap.add_argument("--only", choices=["fixtures", "ref_vectors", "projection", "configs"], default=None,
                    help="regenerate one group only")
    a = ap.parse_args()
    if a.only == "configs":
        config_goldens()
        return
    if not a.ref:
        ap.error("no reference checkout: pass --ref <path> or set P3D_REFERENCE")
    build(a.ref)
    if a.only in (None, "fixtures"):
        run_fixtures()
    if a.only in (None, "ref_vectors"):
        ref_vectors()
    if a.only in (None, "projection"):
        projection_vectors()
    if a.only is None:
        config_goldens()


if __name__ == "__main__":
    main()
