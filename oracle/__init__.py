"""Test infrastructure: CPU oracle for the sparse-voxel SLat hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package.  The product (pixal3d.cpp_b200) never imports it.
"""
