"""CUDA sources of the sandmuon_b200 engine and their build script."""
