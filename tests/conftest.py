"""pytest configuration: import paths and the `gpu` marker.

Tests marked `gpu` need a B200 (sm_100a) and call the CUDA kernels through
libvjattn.so; everything else runs on CPU (`-m "not gpu"`)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "vllm-jax_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libvjattn.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")
