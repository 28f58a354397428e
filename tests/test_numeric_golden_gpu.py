"""CUDA kernels against fixtures produced by the reference's OWN code.

Same fixtures as tests/test_numeric_golden.py (tests/golden/numerics.npz,
written by running vllm-jax's attention(), apply_rope, _update_kv_cache and
the two *_reference functions under a numpy JAX stand-in), now compared with
K3 (RoPE, slot scatter, q scaling), K2 (decode) and K1 (prefill) through the
drop-in boundary `attention(kv_cache, q, k, v, metadata)`. Tolerances:
bit-exact for RoPE and slot writes; attention max-abs <= 2e-2, mean-abs <= 2e-3.
"""
import os
import sys

import ml_dtypes
import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))

import det_inputs as di                      # noqa: E402

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "numerics.npz")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def g(z, key):
    return z[key].view(ml_dtypes.bfloat16).astype(np.float32)


def T(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).cuda()


def I(x):
    return torch.from_numpy(np.asarray(x, np.int32)).cuda()


def N(t):
    return t.float().cpu().numpy()


def close(got, want, rows=None):
    e = np.abs(got - want)
    if rows is not None:
        e = e[rows]
    assert e.max() <= MAX_ABS and e.mean() <= MEAN_ABS, (e.max(), e.mean())


def test_k3_rope_bit_exact_vs_reference(gold):
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope
    x, pos = di.rope_inputs()
    cache = torch.zeros(2, 4, 16, 1, 128, dtype=torch.bfloat16, device="cuda")
    slots = torch.full((len(pos),), -1, dtype=torch.int32, device="cuda")
    q_out, k_out = kv_store_qknorm_rope(T(x), T(x[:, :1]), T(x[:, :1]), cache, slots, I(pos),
                                        norm=False, rope=True, wrap_negative_slots=False,
                                        return_k=True)
    torch.cuda.synchronize()
    want = g(gold, "rope")
    np.testing.assert_array_equal(N(q_out), want)
    np.testing.assert_array_equal(N(k_out), want[:, :1])


def test_k3_update_kv_cache_bit_exact_vs_reference(gold):
    from vllm_b200.kernels.kv_store import update_kv_cache
    cache, slots, k, v = di.kv_update_inputs()
    dc = T(cache)
    update_kv_cache(dc, I(slots), T(k), T(v))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(N(dc), g(gold, "kv_update"))


def test_decode_attention_boundary_vs_reference(gold):
    """attention() with decode metadata: slot writes, q / bf16(sqrt(128)) in
    bf16, K2 with scale 1 -- against the reference's default (Pallas) path,
    its jnp path and paged_attention_reference."""
    from vllm_b200.model.qwen3 import DecodeAttentionMetadata, attention
    d = di.decode_inputs()
    kv = T(d["kv_cache"])
    meta = DecodeAttentionMetadata(input_positions=I(d["positions"]),
                                   slot_mapping=I(d["slot_mapping"]),
                                   block_tables=I(d["block_tables"]),
                                   context_lens=I(d["context_lens"]))
    kv, out = attention(kv, T(d["q"]), T(d["k"]), T(d["v"]), meta)
    torch.cuda.synchronize()
    got = N(out)
    close(got, g(gold, "decode_pallas"))
    close(got, g(gold, "decode_jnp"))
    close(got, g(gold, "decode_refimpl"), rows=d["context_lens"] > 0)
    assert not np.any(got[d["context_lens"] == 0])
    flat = N(kv).reshape(2, -1, 8, 128)
    np.testing.assert_array_equal(flat[:, gold["decode_kv_written_slots"]],
                                  g(gold, "decode_kv_written"))


def test_prefill_attention_boundary_vs_reference(gold):
    """attention() with prefill metadata (4 seats, 3 sequences, bucket-padded
    128 tokens): q * bf16(1/sqrt(128)) in bf16, K1 with scale 1 -- against the
    reference's jnp path, prefill_paged_attention_reference, and the Pallas
    kernel on the rows it computes correctly (each sequence's first q block)."""
    from vllm_b200.model.qwen3 import PrefillAttentionMetadata, attention
    p = di.prefill_inputs()
    cu = I(p["cu_seqlens"])
    mx = max(di.PREFILL_LENS)
    meta = PrefillAttentionMetadata(input_positions=I(p["positions"]),
                                    slot_mapping=I(p["slot_mapping"]),
                                    block_tables=I(p["block_tables"]), cu_seqlens_q=cu,
                                    cu_seqlens_k=cu, max_seqlen_q=mx, max_seqlen_k=mx,
                                    max_seqlen_bucket=p["max_seqlen_bucket"])
    kv, out = attention(T(p["kv_cache"]), T(p["q"]), T(p["k"]), T(p["v"]), meta)
    torch.cuda.synchronize()
    got = N(out)
    close(got, g(gold, "prefill_jnp"))
    close(got, g(gold, "prefill_refimpl"))
    close(got, g(gold, "prefill_pallas_first_block"), rows=gold["prefill_first_block_rows"])
    assert not np.any(got[p["num_tokens"]:])
