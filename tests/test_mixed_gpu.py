"""vj_paged_attention_mixed: a chunked-prefill step's attention in one launch.

Decode rows (one new token each, some with contexts long enough to be split
across chunks) and prompt chunks after a cached prefix, packed decode rows
first and bucket-padded, are checked against the CPU oracle
(oracle.attention.decode_attention / prefill_attention) and against the two
separate launches (vj_paged_decode + vj_paged_prefill) at the north-star bf16
bound (max-abs 2e-2, mean-abs 2e-3); padding rows must be 0. A second call
that reuses the decode split plan (the later layers of a step) is checked too.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _case(Hq, Hkv, dec_ctx, chunks, pad, seed):
    """chunks: list of (prefix, new). Returns numpy and device tensors."""
    rng = np.random.default_rng(seed)
    bs, D = 16, 128
    nd = len(dec_ctx)
    ctx = list(dec_ctx) + [p + n for p, n in chunks]
    S = len(ctx)
    pages = [(c + bs - 1) // bs for c in ctx]
    nb = sum(pages) + 5
    perm = rng.permutation(nb).astype(np.int32)
    width = max(pages) + 1
    bt = np.full((S, width), -1, np.int32)
    o = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[o:o + p]
        o += p
    cu = [0]
    for s in range(S):
        cu.append(cu[-1] + (1 if s < nd else chunks[s - nd][1]))
    T = cu[-1] + pad
    q = bf16(rng.standard_normal((T, Hq, D)))
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, D)))
    t = lambda x, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(x)).to(dt).cuda()
    dev = dict(q=t(q), cache=t(cache), bt=t(bt, torch.int32),
               cu=t(np.asarray(cu, np.int32), torch.int32),
               ctx=t(np.asarray(ctx, np.int32), torch.int32))
    host = dict(q=q, cache=cache, bt=bt, cu=np.asarray(cu), ctx=np.asarray(ctx), nd=nd,
                maxq=max([n for _, n in chunks] + [1]), T=T)
    return host, dev


def _oracle(h, scale):
    nd, q, kc, vc = h["nd"], h["q"], h["cache"][0], h["cache"][1]
    out = np.zeros_like(q)
    if nd:
        out[:nd] = oatt.decode_attention(q[:nd], kc, vc, h["bt"][:nd], h["ctx"][:nd], scale)
    S = len(h["ctx"])
    if S > nd:
        pre = oatt.prefill_attention(q, kc, vc, h["bt"][nd:], h["cu"][nd:], h["ctx"][nd:], scale)
        out[nd:h["cu"][-1]] = pre[nd:h["cu"][-1]]
    return out


def _close(got, want):
    e = np.abs(got - want)
    assert e.max() <= MAX_ABS and e.mean() <= MEAN_ABS, (e.max(), e.mean())


@pytest.mark.parametrize("Hq,Hkv,dec_ctx,chunks,pad", [
    (32, 8, [17, 700, 5000, 33, 2500], [(0, 130), (512, 64), (1000, 300)], 7),
    (32, 8, [], [(0, 200), (300, 17)], 0),                 # chunks only
    (32, 8, [40, 9000, 1], [], 3),                         # decode rows only
    (4, 1, [100, 3000, 60] * 20, [(2000, 256), (0, 1000)], 1),   # TP-8 shard, g = 4
    (64, 8, [1500, 12], [(64, 129)], 0),                   # 32B heads, g = 8
])
def test_mixed_launch_vs_oracle_and_separate_launches(Hq, Hkv, dec_ctx, chunks, pad):
    from vllm_b200.kernels.decode_paged_attention import paged_decode
    from vllm_b200.kernels.prefill_paged_attention import (paged_attention_mixed,
                                                           paged_prefill, pipeline_error)
    h, d = _case(Hq, Hkv, dec_ctx, chunks, pad, seed=len(dec_ctx) * 7 + Hq)
    scale = 1.0 / math.sqrt(128)
    nd, S = h["nd"], len(h["ctx"])
    from vllm_b200 import _native
    ws = torch.empty(max(16, _native.load().vj_paged_attention_mixed_workspace_size(nd, Hq, 128, 0)),
                     dtype=torch.uint8, device="cuda")
    out = torch.full_like(d["q"], float("nan"))
    paged_attention_mixed(d["q"], d["cache"], d["bt"], d["cu"], d["ctx"], nd, h["maxq"],
                          scale, out=out, workspace=ws)
    # the separate launches of the same step
    sep = torch.zeros_like(d["q"])
    if nd:
        paged_decode(d["q"][:nd], d["cache"], d["bt"][:nd], d["ctx"][:nd], scale,
                     out=sep[:nd])
    if S > nd:
        paged_prefill(d["q"], d["cache"], d["bt"][nd:], d["cu"][nd:], d["ctx"][nd:],
                      max_seqlen_q=h["maxq"], scale=scale, out=sep)
    torch.cuda.synchronize()
    assert not pipeline_error()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert not np.any(got[h["cu"][-1]:])                      # padding rows are 0
    _close(got, _oracle(h, scale))
    _close(got, sep.float().cpu().numpy())
    # later layer of the step: same rows, plan reused, new q
    q2 = torch.flip(d["q"], dims=[2]).contiguous()
    out2 = torch.full_like(q2, float("nan"))
    paged_attention_mixed(q2, d["cache"], d["bt"], d["cu"], d["ctx"], nd, h["maxq"], scale,
                          out=out2, workspace=ws, reuse_plan=True)
    torch.cuda.synchronize()
    h2 = dict(h, q=q2.float().cpu().numpy())
    _close(out2.float().cpu().numpy(), _oracle(h2, scale))


def test_mixed_launch_rejects_bad_arguments():
    from vllm_b200.kernels.prefill_paged_attention import paged_attention_mixed
    q = torch.zeros(4, 32, 128, dtype=torch.bfloat16, device="cuda")
    cache = torch.zeros(2, 8, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(2, 4, dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 1, 4], dtype=torch.int32, device="cuda")
    ctx = torch.tensor([1, 3], dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        paged_attention_mixed(q, cache, bt, cu, ctx, 3, 3)     # num_decode > num_seqs
    with pytest.raises(ValueError):
        paged_attention_mixed(q, cache, bt[:1], cu, ctx, 1, 3)  # one table row short
