"""Pixal3D sparse-voxel SLat hot path, B200-native (see pixal3d.cpp_b200)."""
