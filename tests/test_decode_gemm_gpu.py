"""Decode-step GEMMs with fused epilogues (vj_decode_gemm, vj_qkv_gemm_kv_store).

* PLAIN: x @ w.T against a torch fp32 matmul rounded to bf16: the two differ
  only by the order of the fp32 sums, so every output is within one bf16 ulp
  of the reference (plus 1e-4 absolute for values that cancel to near zero); the same
  call is bit-identical when repeated (split partials are summed in a fixed
  order) and for every explicit split count the same within the tolerance.
* SWIGLU: against vj_silu_mul applied to this library's own PLAIN projection
  of [gate; up] (same tiles, same sums): bit-exact.
* QKV + K3: against this library's PLAIN qkv projection followed by
  vj_kv_store_qknorm_rope (bit-exact: the epilogue runs K3's row code) and the
  CPU oracle of K3 (oracle/kv_store.py) on those projections (bit-exact),
  with negative (wrapping) and out-of-range (dropped) slots and positions past
  the RoPE table.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).cuda()


def _ulp_close(got: torch.Tensor, ref32: torch.Tensor):
    """got (bf16) within one bf16 ulp of the fp32 reference, plus 1e-4 absolute
    for outputs that cancel to near zero (sums of ~1 whose fp32 rounding,
    tensor core or not, leaves ~1e-6 absolute: cuBLAS's bf16 GEMM shows the
    same)."""
    g = got.float()
    ulp = torch.abs(ref32) * 2.0 ** -7 + 1e-4
    err = torch.abs(g - ref32)
    bad = err > ulp
    assert not bad.any(), (float(err.max()), int(bad.sum()))


@pytest.mark.parametrize("rows,n,k", [
    (1, 4096, 4096), (7, 6144, 4096), (128, 4096, 4096), (200, 1024, 12288),
    (512, 6144, 4096), (33, 768, 512), (64, 9472, 1024),
])
def test_plain_vs_fp32(rows, n, k):
    from vllm_b200.kernels.gemm import decode_gemm
    x = _rand((rows, k), 1, 1.0)
    w = _rand((n, k), 2, 0.02)
    ref = x.float() @ w.float().T
    out = decode_gemm(x, w)
    torch.cuda.synchronize()
    _ulp_close(out, ref)
    again = decode_gemm(x, w)
    torch.cuda.synchronize()
    assert torch.equal(out, again)                  # fixed split order: reproducible


@pytest.mark.parametrize("rows,splits", [(96, 1), (96, 2), (96, 5), (96, 32),
                                         (40, 2), (40, 3), (40, 8), (40, 32), (5, 4)])
def test_plain_explicit_splits(rows, splits):
    """<= 64 rows and <= 8 splits: the splits of a tile are one cluster and
    reduce through distributed shared memory; otherwise through the
    workspace. Same sums in the same order either way."""
    from vllm_b200.kernels.gemm import decode_gemm
    x = _rand((rows, 4096), 3)
    w = _rand((1024, 4096), 4, 0.02)
    ref = x.float() @ w.float().T
    out = decode_gemm(x, w, splits=splits)
    torch.cuda.synchronize()
    _ulp_close(out, ref)
    if rows <= 64 and splits <= 8:
        glob = decode_gemm(x, w, splits=splits + 24)   # > 8: the workspace path
        torch.cuda.synchronize()
        _ulp_close(glob, ref)


def test_plain_strided_x_and_out():
    """x a column slice of a wider buffer, out a row slice of a wider one."""
    from vllm_b200.kernels.gemm import decode_gemm
    big = _rand((40, 4096 + 64), 5)
    x = big[:, 64:]
    w = _rand((512, 4096), 6, 0.02)
    dst = torch.zeros((40, 1024), dtype=torch.bfloat16, device="cuda")
    decode_gemm(x, w, out=dst[:, 256:768])
    torch.cuda.synchronize()
    _ulp_close(dst[:, 256:768], x.float() @ w.float().T)
    assert not dst[:, :256].any() and not dst[:, 768:].any()


@pytest.mark.parametrize("rows,inter,k", [(1, 12288, 4096), (50, 3072, 1024),
                                          (128, 1536, 4096), (300, 1024, 512)])
def test_swiglu_vs_plain_then_silu_mul(rows, inter, k):
    from vllm_b200.kernels.fused import silu_mul
    from vllm_b200.kernels.gemm import decode_gemm
    x = _rand((rows, k), 7)
    w = _rand((2 * inter, k), 8, 0.05)
    fused = decode_gemm(x, w, "swiglu")
    gu = decode_gemm(x, w)                          # same tiles and sums
    ref = silu_mul(gu)
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)


def _qkv_case(T, Hq, Hkv, hidden, nb=64, bs=16, seed=0):
    D = 128
    x = _rand((T, hidden), seed + 1)
    w = _rand(((Hq + 2 * Hkv) * D, hidden), seed + 2, 0.03)
    qn = _rand((D,), seed + 3, 0.3) + 1.0
    kn = _rand((D,), seed + 4, 0.3) + 1.0
    cache = _rand((2, nb, bs, Hkv, D), seed + 5)
    g = torch.Generator(device="cpu").manual_seed(seed)
    slots = torch.randperm(nb * bs - 1, generator=g)[:T].to(torch.int32)  # last slot: -1 only
    if T > 3:
        slots[1] = -1                        # wraps to the pool's last slot
        slots[2] = nb * bs + 5               # dropped
    pos = torch.randint(0, 6000, (T,), generator=g).to(torch.int32)
    if T > 4:
        pos[3] = 50000                       # past the 4096-entry table: computed in-kernel
    return x, w, qn, kn, cache, slots.cuda(), pos.cuda()


@pytest.mark.parametrize("T,Hq,Hkv,hidden,q_scale", [
    (1, 32, 8, 4096, None), (37, 32, 8, 4096, "div"), (128, 32, 8, 4096, "mul"),
    (200, 4, 1, 4096, None), (64, 16, 8, 1024, "div"),
])
def test_qkv_kv_store_vs_plain_then_k3(T, Hq, Hkv, hidden, q_scale):
    from vllm_b200.kernels.gemm import decode_gemm, qkv_gemm_kv_store
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope, rope_table
    x, w, qn, kn, cache, slots, pos = _qkv_case(T, Hq, Hkv, hidden, seed=T + Hq)
    table = rope_table(x.device, 1e6, 4096)
    c_fused = cache.clone()
    q_fused = qkv_gemm_kv_store(x, w, c_fused, slots, pos, qn, kn, Hq, eps=1e-6,
                                rope_theta=1e6, q_scale=q_scale, table=table)
    qkv = decode_gemm(x, w)
    D = 128
    q, k, v = torch.split(qkv, [Hq * D, Hkv * D, Hkv * D], -1)
    c_ref = cache.clone()
    q_ref = kv_store_qknorm_rope(q.reshape(T, Hq, D).contiguous(), k.reshape(T, Hkv, D).contiguous(),
                                 v.reshape(T, Hkv, D).contiguous(), c_ref, slots, pos, qn, kn,
                                 eps=1e-6, rope_theta=1e6, q_scale=q_scale, table=table)
    torch.cuda.synchronize()
    assert torch.equal(q_fused, q_ref)
    assert torch.equal(c_fused, c_ref)

    # the CPU oracle of K3 on the same projections
    from oracle import kv_store as ork
    f = lambda t: t.float().cpu().numpy()
    kc, vc = f(cache[0]).copy(), f(cache[1]).copy()
    q_or, _ = ork.kv_store_qknorm_rope(f(q).reshape(T, Hq, D), f(k).reshape(T, Hkv, D),
                                       f(v).reshape(T, Hkv, D), f(qn), f(kn),
                                       pos.cpu().numpy(), slots.cpu().numpy(), kc, vc,
                                       eps=1e-6, rope_theta=1e6, q_scale=q_scale)
    assert np.array_equal(f(q_fused), q_or)
    assert np.array_equal(f(c_fused[0]), kc) and np.array_equal(f(c_fused[1]), vc)


def test_rejects_bad_arguments():
    from vllm_b200.kernels.gemm import decode_gemm
    x = _rand((4, 100), 1)
    w = _rand((128, 100), 2)
    with pytest.raises(Exception):
        decode_gemm(x, w)                               # k not a multiple of 64
    x = _rand((4, 128), 1)
    w = _rand((100, 128), 2)
    with pytest.raises(Exception):
        decode_gemm(x, w)                               # n not a multiple of 128
    with pytest.raises(ValueError):
        decode_gemm(x, _rand((128, 128), 3), mode="gelu")


@pytest.mark.parametrize("rows", [1, 16, 100, 300])
def test_packed_weight_tiles_bit_identical(rows):
    """TiledWeight (vj_pack_weight_tiles + bulk-copied stages) gives the same
    bits as the row-major weight read through tensor maps, for all modes."""
    from vllm_b200.kernels.gemm import TiledWeight, decode_gemm, qkv_gemm_kv_store
    from vllm_b200.kernels.kv_store import rope_table
    x = _rand((rows, 1024), 11)
    w = _rand((1536, 1024), 12, 0.03)
    assert torch.equal(decode_gemm(x, w), decode_gemm(x, TiledWeight(w)))
    assert torch.equal(decode_gemm(x, w, "swiglu"), decode_gemm(x, TiledWeight(w, "swiglu"), "swiglu"))
    with pytest.raises(ValueError):
        decode_gemm(x, TiledWeight(w), "swiglu")        # packed for the other mode
    x, wq, qn, kn, cache, slots, pos = _qkv_case(rows, 8, 2, 1024, seed=rows)
    table = rope_table(x.device, 1e6, 4096)
    c1, c2 = cache.clone(), cache.clone()
    q1 = qkv_gemm_kv_store(x, wq, c1, slots, pos, qn, kn, 8, table=table)
    q2 = qkv_gemm_kv_store(x, TiledWeight(wq), c2, slots, pos, qn, kn, 8, table=table)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(c1, c2)


@pytest.mark.parametrize("rows,splits", [(16, 2), (61, 4), (1, 8)])
def test_cluster_reduction_many_tiles_all_modes(rows, splits):
    """Cluster split-K with more weight tiles than clusters (each cluster
    walks several tiles: its partial buffer is reused once every peer has
    read it), in all three epilogues; against the workspace reduction of the
    same split count (> 8 forces it) or the plain path."""
    from vllm_b200.kernels.fused import silu_mul
    from vllm_b200.kernels.gemm import decode_gemm, qkv_gemm_kv_store
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope, rope_table
    x = _rand((rows, 4096), 21)
    w = _rand((24576, 4096), 22, 0.02)                  # 192 weight tiles
    ref = x.float() @ w.float().T
    out = decode_gemm(x, w, splits=splits)
    torch.cuda.synchronize()
    _ulp_close(out, ref)
    sw = decode_gemm(x, w, "swiglu", splits=splits)
    torch.cuda.synchronize()
    _ulp_close(sw.float(), silu_mul(out).float())      # same arithmetic on ~equal inputs
    x, wq, qn, kn, cache, slots, pos = _qkv_case(rows, 32, 8, 4096, seed=rows + 100)
    table = rope_table(x.device, 1e6, 4096)
    c1, c2 = cache.clone(), cache.clone()
    q1 = qkv_gemm_kv_store(x, wq, c1, slots, pos, qn, kn, 32, table=table, splits=splits)
    qkv = decode_gemm(x, wq, splits=splits)
    D = 128
    q, k, v = torch.split(qkv, [32 * D, 8 * D, 8 * D], -1)
    q2 = kv_store_qknorm_rope(q.reshape(rows, 32, D).contiguous(),
                              k.reshape(rows, 8, D).contiguous(),
                              v.reshape(rows, 8, D).contiguous(), c2, slots, pos, qn, kn,
                              table=table)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(c1, c2)  # same splits, same sums
