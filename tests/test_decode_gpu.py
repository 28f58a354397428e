"""K2 split-KV paged decode on the GPU vs the CPU oracle.

Tolerance: max-abs error <= 2e-2, mean-abs error <= 2e-3
against the fp32 oracle on bf16 inputs."""
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


def _make(B, Hq, Hkv, lens, nb, bs, width, seed):
    rng = np.random.default_rng(seed)
    D = 128
    q = bf16(rng.standard_normal((B, Hq, D)))
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, D)))
    perm = rng.permutation(nb)
    bt = np.full((B, width), -1, np.int32)
    used = 0
    for b, L in enumerate(lens):
        n = (L + bs - 1) // bs
        bt[b, :n] = perm[used:used + n]
        used += n
    assert used <= nb
    return q, cache, bt, np.asarray(lens, np.int32)


def _check(out, ref):
    err = np.abs(out - ref)
    assert err.max() <= MAX_ABS, f"max abs err {err.max()}"
    assert err.mean() <= MEAN_ABS, f"mean abs err {err.mean()}"


@pytest.mark.parametrize("B,Hq,Hkv,bs,lens", [
    (1, 32, 8, 16, [1]),
    (4, 16, 8, 16, [17, 64, 129, 300]),              # 0.6B shapes (C1 prompts)
    (5, 32, 8, 16, [0, 15, 16, 17, 1000]),           # empty + page edges
    (3, 64, 8, 16, [4000, 33, 2048]),                # 32B heads (g=8)
    (6, 4, 1, 16, [700, 1, 2, 3000, 48, 129]),       # TP-8 shard
    (4, 32, 8, 32, [31, 32, 33, 2500]),              # block_size 32
    (2, 16, 4, 64, [64, 5000]),                      # block_size 64
])
def test_paged_decode_matches_oracle(B, Hq, Hkv, bs, lens):
    from vllm_b200.kernels.decode_paged_attention import paged_decode
    nb = sum((L + bs - 1) // bs for L in lens) + 7
    width = max((L + bs - 1) // bs for L in lens) + 3
    q, cache, bt, ln = _make(B, Hq, Hkv, lens, nb, bs, width, seed=B * 100 + Hq)
    scale = 1.0 / math.sqrt(128)
    ref = oatt.decode_attention(q, cache[0], cache[1], bt, ln, scale)
    # the output starts as NaN: every row (zero-length ones included) must be written
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device="cuda")
    out = paged_decode(_t(q), _t(cache), _t(bt, torch.int32), _t(ln, torch.int32), scale,
                       out=out)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    _check(got, ref)
    for b, L in enumerate(lens):
        if L == 0:
            assert np.all(got[b] == 0)


def test_paged_decode_many_splits_and_small_chunks():
    """Long contexts force multi-chunk combine; max_chunks bounds the split."""
    from vllm_b200.kernels.decode_paged_attention import paged_decode
    lens = [9000, 12000, 130, 7777]
    bs, Hq, Hkv = 16, 32, 8
    nb = sum((L + bs - 1) // bs for L in lens)
    width = 760
    q, cache, bt, ln = _make(4, Hq, Hkv, lens, nb, bs, width, seed=11)
    ref = oatt.decode_attention(q, cache[0], cache[1], bt, ln, 1 / math.sqrt(128))
    for max_chunks in (0, 8, 64):
        out = paged_decode(_t(q), _t(cache), _t(bt, torch.int32), _t(ln, torch.int32),
                           max_chunks=max_chunks)
        torch.cuda.synchronize()
        _check(out.float().cpu().numpy(), ref)


def test_decode_paged_attention_reference_api():
    """Reference signature: pages [Hkv, total_pages, page_size, D], q pre-scaled."""
    from vllm_b200.kernels.decode_paged_attention import decode_paged_attention
    B, Hq, Hkv, bs = 3, 32, 8, 16
    lens = [100, 1, 513]
    nb = 80
    q, cache, bt, ln = _make(B, Hq, Hkv, lens, nb, bs, 64, seed=5)
    # the reference scales q in bf16 before the kernel (vllm/model/qwen3.py:207)
    q_scaled = bf16(q / np.float32(bf16(np.sqrt(np.float32(128)))))
    k_pages = np.ascontiguousarray(cache[0].transpose(2, 0, 1, 3))
    v_pages = np.ascontiguousarray(cache[1].transpose(2, 0, 1, 3))
    ref = oatt.decode_attention(q_scaled, cache[0], cache[1], np.where(bt >= 0, bt, 0), ln, 1.0)
    out = decode_paged_attention(_t(q_scaled), _t(k_pages), _t(v_pages),
                                 _t(np.where(bt >= 0, bt, 0), torch.int32), _t(ln, torch.int32),
                                 k_splits=16)
    torch.cuda.synchronize()
    _check(out.float().cpu().numpy(), ref)
    with pytest.raises(ValueError, match="same batch size"):
        decode_paged_attention(_t(q_scaled), _t(k_pages), _t(v_pages),
                               _t(bt[:2], torch.int32), _t(ln, torch.int32))
    with pytest.raises(ValueError, match="divisible"):
        decode_paged_attention(_t(q_scaled[:, :30]), _t(k_pages), _t(v_pages),
                               _t(bt, torch.int32), _t(ln, torch.int32))


def test_paged_decode_large_batch_properties():
    """C3-like shape at reduced size: outputs are convex combinations of V rows,
    so every output lies inside [min V, max V] of its sequence, and a rerun is
    bitwise identical (the split plan is deterministic for fixed lengths)."""
    from vllm_b200.kernels.decode_paged_attention import paged_decode
    rng = np.random.default_rng(0)
    B, Hq, Hkv, bs = 64, 32, 8, 16
    lens = np.round(np.exp(rng.uniform(np.log(512), np.log(8192), B))).astype(np.int32)
    nb = int(sum((L + bs - 1) // bs for L in lens))
    width = 512
    q, cache, bt, ln = _make(B, Hq, Hkv, list(lens), nb, bs, width, seed=1)
    dq, dc, dbt, dl = _t(q), _t(cache), _t(bt, torch.int32), _t(ln, torch.int32)
    o1 = paged_decode(dq, dc, dbt, dl)
    o2 = paged_decode(dq, dc, dbt, dl)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    ref = oatt.decode_attention(q[:8], cache[0], cache[1], bt[:8], ln[:8], 1 / math.sqrt(128))
    _check(o1[:8].float().cpu().numpy(), ref)
    vmax = float(np.abs(cache[1]).max())
    assert float(o1.float().abs().max()) <= vmax + 1e-2


def test_planned_decode_reuses_the_plan_of_the_first_call():
    """vj_paged_decode_planned (the layers after the first of a decode step)
    skips the planning launch and gives the oracle's result for new q, K and
    V with the same lengths, several times in a row."""
    from vllm_b200.kernels.decode_paged_attention import decode_workspace_bytes, paged_decode
    B, Hq, Hkv, bs = 6, 32, 8, 16
    lens = [0, 700, 33, 5000, 16, 2049]
    nb = sum((L + bs - 1) // bs for L in lens) + 7
    width = max((L + bs - 1) // bs for L in lens) + 3
    ws = torch.empty(decode_workspace_bytes(B, Hq), dtype=torch.uint8, device="cuda")
    scale = 1.0 / math.sqrt(128)
    for layer in range(4):
        q, cache, bt, ln = _make(B, Hq, Hkv, lens, nb, bs, width, seed=77 + layer)
        ref = oatt.decode_attention(q, cache[0], cache[1], bt, ln, scale)
        out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device="cuda")
        out = paged_decode(_t(q), _t(cache), _t(bt, torch.int32), _t(ln, torch.int32), scale,
                           out=out, workspace=ws, reuse_plan=layer > 0)
        torch.cuda.synchronize()
        _check(out.float().cpu().numpy(), ref)
