"""The C-ABI library loads on CPU, exports every symbol include/vjattn.h declares,
and rejects bad arguments before touching the GPU."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def _declared_symbols():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(vj_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    syms = _declared_symbols()
    for required in ("vj_kv_store_qknorm_rope", "vj_paged_decode", "vj_get_last_error"):
        assert required in syms


def test_library_exports_every_declared_symbol():
    from vllm_b200 import _native
    lib = _native.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), f"libvjattn.so does not export {name}"
        assert name in _native.PROTOTYPES, f"no ctypes prototype for {name}"


def test_validation_without_gpu():
    from vllm_b200 import _native
    lib = _native.load()
    assert lib.vj_version() >> 16 == 2
    # head_dim 64 is rejected before any CUDA call
    st = lib.vj_kv_store_qknorm_rope(None, 1, 1, None, None, None, 1, None, None, 16, 16,
                                     4, 0, 2, 64, 4, 16, 4096, 256, 128, 0, 0, 0, None, 0,
                                     1e-6, 1e6, 0, None)
    assert st == _native.VJ_ERR_UNSUPPORTED
    assert b"head_dim" in lib.vj_get_last_error()
    # both q scalings at once are rejected
    st = lib.vj_kv_store_qknorm_rope(None, 1, 1, None, None, None, 1, None, None, 16, 16,
                                     4, 0, 2, 128, 4, 16, 4096, 256, 128, 0, 0, 0, None, 0,
                                     1e-6, 1e6, _native.VJ_KV_QSCALE_DIV_SQRT_D
                                     | _native.VJ_KV_QSCALE_MUL_RSQRT_D, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT
    # a misaligned rope table is rejected
    st = lib.vj_kv_store_qknorm_rope(None, 16, 16, None, None, 16, 16, None, None, 16, 16,
                                     4, 0, 2, 128, 4, 16, 4096, 256, 128, 0, 0, 0, 8, 10,
                                     1e-6, 1e6, _native.VJ_KV_ROPE, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT
    assert b"rope_table" in lib.vj_get_last_error()
    assert lib.vj_rope_table_bytes(1000, 128) == 1000 * 64 * 4
    assert lib.vj_rope_table_bytes(1000, 64) == 0
    assert lib.vj_rope_table_build(None, 10, 128, 1e6, None) == _native.VJ_ERR_INVALID_ARGUMENT
    st = lib.vj_paged_decode(1, 1, 1, 1, 1, 1, 2, 12, 8, 128, 10, 16, 4, 4, 16 * 1024, 1024,
                             128, 0.1, 0, None, 0, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT
    assert b"divisible" in lib.vj_get_last_error()
    # workspace too small
    st = lib.vj_paged_decode(1, 1, 1, 1, 1, 1, 2, 32, 8, 128, 10, 16, 4, 4, 16 * 1024, 1024,
                             128, 0.1, 0, 16, 8, None)
    assert st == _native.VJ_ERR_WORKSPACE
    assert lib.vj_paged_decode_workspace_size(256, 32, 128, 0) > 0
    assert lib.vj_paged_decode_workspace_size(256, 32, 64, 0) == 0
    # decode GEMMs: qkv of Qwen3-8B at 128 rows splits K in 3 (48 tiles x 3 =
    # 144 units on 148 SMs): the 64 KB ticket area + 48 x 3 fp32 128x128 partials
    assert lib.vj_decode_gemm_workspace_size(128, 6144, 4096, _native.VJ_GEMM_PLAIN, 0) == \
        65536 + 48 * 3 * 128 * 128 * 4
    assert lib.vj_decode_gemm_workspace_size(128, 6144, 4096, _native.VJ_GEMM_PLAIN, 1) == 65536
    assert lib.vj_decode_gemm_workspace_size(128, 6144, 100, _native.VJ_GEMM_PLAIN, 0) == 0
    st = lib.vj_decode_gemm(16, 0, 16, 0, 16, 0, 4, 256, 100, _native.VJ_GEMM_PLAIN, 0, 16,
                            1 << 20, None, None)
    assert st == _native.VJ_ERR_UNSUPPORTED and b"multiple of 64" in lib.vj_get_last_error()
    st = lib.vj_decode_gemm(16, 0, 16, 0, 16, 0, 4, 256, 128, 7, 0, 16, 1 << 20, None, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT
    st = lib.vj_decode_gemm(16, 0, 16, 0, 16, 0, 4, 256, 128, _native.VJ_GEMM_PLAIN, 0, 16, 64,
                            None, None)
    assert st == _native.VJ_ERR_WORKSPACE
    st = lib.vj_decode_gemm(16, 0, 16, 5, 16, 0, 4, 256, 128, _native.VJ_GEMM_PLAIN, 0, 256,
                            1 << 20, None, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT and b"weight_layout" in lib.vj_get_last_error()
    assert lib.vj_pack_weight_tiles(16, 32, 100, 64, 0, None) == _native.VJ_ERR_UNSUPPORTED
    assert lib.vj_pack_weight_tiles(16, 16, 128, 64, 0, None) == _native.VJ_ERR_INVALID_ARGUMENT
    st = lib.vj_qkv_gemm_kv_store(16, 0, 16, 0, 16, 16, 16, 16, 16, 16, 16, 4, 4096, 32, 8, 64,
                                  16, 16, 4096, 256, 128, None, 0, 1e-6, 1e6, 0, 0, 16, 1 << 20,
                                  None, None)
    assert st == _native.VJ_ERR_UNSUPPORTED and b"head_dim" in lib.vj_get_last_error()


def test_no_cpu_fallback_for_cpu_tensors():
    torch = pytest.importorskip("torch")
    from vllm_b200.kernels.decode_paged_attention import paged_decode
    q = torch.zeros(1, 32, 128, dtype=torch.bfloat16)
    cache = torch.zeros(2, 4, 16, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        paged_decode(q, cache, torch.zeros(1, 4, dtype=torch.int32),
                     torch.ones(1, dtype=torch.int32))
