"""K3 (q/k RMSNorm + RoPE + KV scatter) on the GPU vs the CPU oracle, bit for bit."""
import numpy as np
import pytest
import torch

from oracle import kv_store as ork
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu


def _bf16_tensor(x, dev="cuda"):
    return torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16).to(dev)


def _np(t):
    return t.float().cpu().numpy()


def _case(T, Hq, Hkv, nb, bs, seed, pos_max=40000, neg_slots=0, dup_slots=False):
    rng = np.random.default_rng(seed)
    D = 128
    q = bf16(rng.standard_normal((T, Hq, D)) * 1.5)
    k = bf16(rng.standard_normal((T, Hkv, D)) * 0.7)
    v = bf16(rng.standard_normal((T, Hkv, D)))
    qw = bf16(1.0 + 0.1 * rng.standard_normal(D))
    kw = bf16(1.0 + 0.1 * rng.standard_normal(D))
    pos = rng.integers(0, pos_max, size=T).astype(np.int32)
    slots = rng.permutation(nb * bs)[:T].astype(np.int32)
    if dup_slots:
        slots[1::2] = slots[0::2][: len(slots[1::2])]
    if neg_slots:
        # bucket padding: identical rows (token id 0 at position 0), all slot -1
        slots[-neg_slots:] = -1
        pos[-neg_slots:] = 0
        k[-neg_slots:] = k[-neg_slots]
        v[-neg_slots:] = v[-neg_slots]
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, D)))
    return q, k, v, qw, kw, pos, slots, cache


@pytest.mark.parametrize("q_scale", [None, "div", "mul"])
@pytest.mark.parametrize("table_positions", [0, 100, 50000])
def test_kv_store_q_scaling_and_rope_table(q_scale, table_positions):
    """The reference's bf16 q scalings, and positions inside / past the end of
    the (cos, sin) table (past the end: computed in the kernel, same bits)."""
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope, rope_table
    q, k, v, qw, kw, pos, slots, cache = _case(257, 32, 8, 32, 16, seed=5, pos_max=45000)
    kc, vc = cache[0].copy(), cache[1].copy()
    q_ref, k_ref = ork.kv_store_qknorm_rope(q, k, v, qw, kw, pos, slots, kc, vc,
                                            eps=1e-6, rope_theta=1e6, q_scale=q_scale)
    dcache = _bf16_tensor(cache)
    table = None
    if table_positions:
        table = rope_table(torch.device("cuda"), 1e6, table_positions)[:table_positions * 64]
    else:
        table = torch.empty(0, dtype=torch.int32, device="cuda")
    q_out, k_out = kv_store_qknorm_rope(_bf16_tensor(q), _bf16_tensor(k), _bf16_tensor(v),
                                        dcache, torch.from_numpy(slots).cuda(),
                                        torch.from_numpy(pos).cuda(), _bf16_tensor(qw),
                                        _bf16_tensor(kw), eps=1e-6, rope_theta=1e6,
                                        return_k=True, q_scale=q_scale, table=table)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_np(q_out), q_ref)
    np.testing.assert_array_equal(_np(k_out), k_ref)
    got = _np(dcache)
    np.testing.assert_array_equal(got[0], kc)
    np.testing.assert_array_equal(got[1], vc)


def test_rope_table_matches_oracle():
    from vllm_b200.kernels.kv_store import rope_table
    n = 70000
    tab = rope_table(torch.device("cuda"), 1e6, n)[:n * 64].view(n, 64).cpu().numpy()
    pos = np.arange(n, dtype=np.int32)
    c, s = ork.rope_cos_sin(pos, 1e6)
    words = tab.view(np.uint32)
    got_c = (words & 0xFFFF).astype(np.uint32) << 16
    got_s = words & 0xFFFF0000
    np.testing.assert_array_equal(got_c.view(np.float32), c)
    np.testing.assert_array_equal(got_s.view(np.float32), s)


@pytest.mark.parametrize("T,Hq,Hkv,nb,bs,neg", [
    (1, 16, 8, 4, 16, 0),
    (37, 16, 8, 8, 16, 3),        # 0.6B heads, padded tokens with slot -1
    (300, 32, 8, 64, 16, 0),      # 8B heads
    (129, 64, 8, 32, 16, 5),      # 32B heads
    (50, 4, 1, 16, 32, 0),        # TP-8 shard, block_size 32
    (33, 8, 1, 16, 16, 2),        # 32B TP-8 shard: k and v rows share a warp
    (700, 12, 2, 64, 16, 0),      # odd q/k/v boundaries in one pass, many tokens
])
def test_kv_store_bit_exact(T, Hq, Hkv, nb, bs, neg):
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope
    q, k, v, qw, kw, pos, slots, cache = _case(T, Hq, Hkv, nb, bs, seed=T, neg_slots=neg)
    kc, vc = cache[0].copy(), cache[1].copy()
    q_ref, k_ref = ork.kv_store_qknorm_rope(q, k, v, qw, kw, pos, slots, kc, vc,
                                            eps=1e-6, rope_theta=1e6)
    dq = _bf16_tensor(q)
    dcache = _bf16_tensor(cache)
    q_out, k_out = kv_store_qknorm_rope(dq, _bf16_tensor(k), _bf16_tensor(v), dcache,
                                        torch.from_numpy(slots).cuda(),
                                        torch.from_numpy(pos).cuda(), _bf16_tensor(qw),
                                        _bf16_tensor(kw), eps=1e-6, rope_theta=1e6,
                                        return_k=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_np(q_out), q_ref)
    np.testing.assert_array_equal(_np(k_out), k_ref)
    got = _np(dcache)
    np.testing.assert_array_equal(got[0], kc)
    np.testing.assert_array_equal(got[1], vc)


def test_update_kv_cache_drop_and_wrap():
    """Plain scatter (qwen3.py:105-111): -1 wraps to the last slot, others drop."""
    from vllm_b200.kernels.kv_store import update_kv_cache
    rng = np.random.default_rng(7)
    nb, bs, Hkv, D, T = 6, 16, 2, 128, 9
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, D)))
    k = bf16(rng.standard_normal((T, Hkv, D)))
    v = bf16(rng.standard_normal((T, Hkv, D)))
    slots = np.array([0, 17, -1, 94, 96, 1000, -7, 5, -200], np.int32)
    kc, vc = cache[0].copy(), cache[1].copy()
    ork.update_kv_cache(kc, vc, slots, k, v)
    dcache = _bf16_tensor(cache)
    update_kv_cache(dcache, torch.from_numpy(slots).cuda(), _bf16_tensor(k), _bf16_tensor(v))
    torch.cuda.synchronize()
    got = _np(dcache)
    np.testing.assert_array_equal(got[0], kc)
    np.testing.assert_array_equal(got[1], vc)
    # slot -1 -> last slot (block 5, offset 15) received token 2's rows
    np.testing.assert_array_equal(got[0, 5, 15], k[2])


def test_kv_store_no_norm_no_rope_is_copy():
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope
    q, k, v, qw, kw, pos, slots, cache = _case(20, 8, 4, 8, 16, seed=3)
    dcache = _bf16_tensor(cache)
    q_out = kv_store_qknorm_rope(_bf16_tensor(q), _bf16_tensor(k), _bf16_tensor(v), dcache,
                                 torch.from_numpy(slots).cuda(), norm=False, rope=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_np(q_out), q)
    flat = _np(dcache)[0].reshape(-1, 4, 128)
    np.testing.assert_array_equal(flat[slots], k)


def test_kv_store_rejects_bad_args():
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope
    k = torch.zeros(4, 2, 64, dtype=torch.bfloat16, device="cuda")
    cache = torch.zeros(2, 4, 16, 2, 64, dtype=torch.bfloat16, device="cuda")
    slots = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(Exception, match="head_dim"):
        kv_store_qknorm_rope(None, k, k, cache, slots, norm=False, rope=False)
    with pytest.raises(ValueError):
        kv_store_qknorm_rope(None, k, k, cache, slots.long(), norm=False, rope=False)


def test_kv_store_no_wait_timed_out():
    """Every call above completed without a staged-kernel wait running out."""
    import ctypes

    from vllm_b200 import _native
    torch.cuda.synchronize()
    n = ctypes.c_int32(-1)
    _native.check(_native.load().vj_kv_store_timeouts(ctypes.byref(n), 0))
    assert n.value == 0
