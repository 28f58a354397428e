"""Torch-facing wrappers of libvjattn (the sm_100a kernels). No CPU fallback."""
