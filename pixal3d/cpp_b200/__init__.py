"""B200-native (sm_100a) sparse-voxel SLat hot path of Pixal3D.cpp.

libp3dcuda.so (built from csrc/ by build.py) holds every kernel behind the C
ABI in include/p3d.h.  `ops` is the torch-tensor front end of that ABI and
`flow` the device-resident SLat flow model / sampler.  There is no CPU or
library fallback: importing `ops` without the built library raises.
"""
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libp3dcuda.so"
HOST_LIB_PATH = Path(__file__).resolve().parent / "libpixal3d_b200.so"
