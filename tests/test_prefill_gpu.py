"""K1 tcgen05 varlen paged prefill on the GPU vs the CPU oracle.

Tolerance: max-abs error <= 2e-2, mean-abs <= 2e-3."""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _t(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).cuda()


def _make(new, prefix, Hq, Hkv, bs, seed, pad=0, extra_blocks=5):
    rng = np.random.default_rng(seed)
    D = 128
    S = len(new)
    ctx = [n + p for n, p in zip(new, prefix)]
    nb = sum((c + bs - 1) // bs for c in ctx) + extra_blocks
    width = max((c + bs - 1) // bs for c in ctx) + 2
    perm = rng.permutation(nb)
    bt = np.full((S, width), -1, np.int32)
    used = 0
    for s, c in enumerate(ctx):
        k = (c + bs - 1) // bs
        bt[s, :k] = perm[used:used + k]
        used += k
    T = sum(new) + pad
    q = bf16(rng.standard_normal((T, Hq, D)))
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, D)))
    cu = np.concatenate([[0], np.cumsum(new)]).astype(np.int32)
    return q, cache, bt, cu, np.asarray(ctx, np.int32)


def _check(got, ref, label=""):
    err = np.abs(got - ref)
    if err.max() > MAX_ABS or err.mean() > MEAN_ABS:
        bad = np.argwhere(err > MAX_ABS)
        rows = np.unique(bad[:, 0])[:10] if len(bad) else []
        heads = np.unique(bad[:, 1])[:10] if len(bad) else []
        raise AssertionError(f"{label} max {err.max():.4g} mean {err.mean():.4g}; "
                             f"{len(bad)} bad elems, rows {rows}, heads {heads}")


CASES = [
    # new tokens, cached prefix, Hq, Hkv, bs
    ([1], [0], 32, 8, 16),
    ([17], [0], 16, 8, 16),
    ([128], [0], 32, 8, 16),
    ([129, 5], [0, 0], 32, 8, 16),
    ([17, 64, 129, 300], [0, 0, 0, 0], 16, 8, 16),        # C1 prompts, 0.6B heads
    ([300, 40], [100, 513], 32, 8, 16),                     # cached prefixes
    ([1000, 77, 512], [0, 2048, 1], 64, 8, 16),             # 32B heads (g = 8)
    ([250, 31], [7, 0], 4, 1, 16),                          # TP-8 shard (g = 4, Hkv = 1)
    ([200, 33], [60, 0], 32, 8, 32),                        # block_size 32
    ([64], [0], 8, 8, 16),                                  # g = 1
]


@pytest.mark.parametrize("new,prefix,Hq,Hkv,bs", CASES)
def test_paged_prefill_matches_oracle(new, prefix, Hq, Hkv, bs):
    from vllm_b200.kernels.prefill_paged_attention import paged_prefill, pipeline_error
    q, cache, bt, cu, ctx = _make(new, prefix, Hq, Hkv, bs, seed=sum(new) + Hq, pad=3)
    scale = 1.0 / math.sqrt(128)
    ref = oatt.prefill_attention(q, cache[0], cache[1], bt, cu, ctx, scale)
    out = paged_prefill(_t(q), _t(cache), _t(bt, torch.int32), _t(cu, torch.int32),
                        _t(ctx, torch.int32), max_seqlen_q=max(new))
    torch.cuda.synchronize()
    assert not pipeline_error()
    got = out.float().cpu().numpy()
    _check(got, ref, f"new={new} prefix={prefix}")
    assert np.all(got[cu[-1]:] == 0)      # bucket padding rows are zero


def test_prefill_reference_api_no_prefix():
    """Reference signature (pages [Hkv, nb, ps, D], cu_seqlens padded to
    max_num_seqs + 1 by repeating the last value, slot -1 padding)."""
    from vllm_b200.kernels.prefill_paged_attention import prefill_paged_attention
    new = [40, 100, 7]
    q, cache, bt, cu, ctx = _make(new, [0, 0, 0], 32, 8, 16, seed=3, pad=109)
    # pad batch to 4 sequences like prepare_prefill (model_runner.py:250-251,255)
    cu4 = np.concatenate([cu, [cu[-1]]]).astype(np.int32)
    bt4 = np.concatenate([bt, np.full((1, bt.shape[1]), -1, np.int32)])
    ref = oatt.prefill_attention(q, cache[0], cache[1], bt, cu, ctx, 1 / math.sqrt(128))
    k_pages = np.ascontiguousarray(cache[0].transpose(2, 0, 1, 3))
    v_pages = np.ascontiguousarray(cache[1].transpose(2, 0, 1, 3))
    T = q.shape[0]
    out = prefill_paged_attention(_t(q), _t(k_pages), _t(v_pages),
                                  _t(np.where(bt4 >= 0, bt4, 0), torch.int32),
                                  _t(cu4, torch.int32), _t(np.full(T, -1), torch.int32),
                                  _t(np.zeros(T), torch.int32), max_seqlen_bucket=128)
    torch.cuda.synchronize()
    _check(out.float().cpu().numpy(), ref, "reference api")
    with pytest.raises(ValueError, match="cu_seqlens"):
        prefill_paged_attention(_t(q), _t(k_pages), _t(v_pages), _t(bt4, torch.int32),
                                _t(cu, torch.int32), None, None, max_seqlen_bucket=128)


def test_prefill_long_sequence_properties():
    """A 4096-token prompt with a 2048 prefix (C2's largest shape): spot rows
    against the oracle and check determinism of a rerun."""
    from vllm_b200.kernels.prefill_paged_attention import paged_prefill
    new, prefix = [4096], [2048]
    q, cache, bt, cu, ctx = _make(new, prefix, 32, 8, 16, seed=9)
    dq, dc, dbt, dcu, dctx = _t(q), _t(cache), _t(bt, torch.int32), _t(cu, torch.int32), \
        _t(ctx, torch.int32)
    o1 = paged_prefill(dq, dc, dbt, dcu, dctx, max_seqlen_q=4096)
    o2 = paged_prefill(dq, dc, dbt, dcu, dctx, max_seqlen_q=4096)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    rows = np.array([0, 1, 31, 32, 1000, 2047, 4000, 4095])
    sub_q = q[rows]
    k = oatt.gather_pages(cache[0], bt[0], int(ctx[0]))
    v = oatt.gather_pages(cache[1], bt[0], int(ctx[0]))
    got = o1.float().cpu().numpy()[rows]
    for i, r in enumerate(rows):
        L = prefix[0] + r + 1
        qh = sub_q[i].reshape(8, 4, 128)
        s = np.einsum("kgd,skd->kgs", qh, k[:L]) / math.sqrt(128)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        o = bf16(np.einsum("kgs,skd->kgd", p, v[:L]).reshape(32, 128))
        _check(got[i], o, f"row {r}")
