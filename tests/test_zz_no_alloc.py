"""vj_paged_decode_noalloc: decode attention for callers that must not allocate.

A caller like an XLA/JAX custom-call handler cannot cudaMalloc (the runtime
owns device memory), so this entry point keeps its scratch in a fixed device
array instead of a caller workspace. These tests call it through the C ABI
(ctypes, no torch wrapper) and check, on two calls in a row, that it matches
the workspace entry point vj_paged_decode and the CPU oracle
(oracle.attention.decode_attention) within the decode tolerance (max-abs
2e-2, mean-abs 2e-3), and that oversized shapes are rejected. The file is
named to be collected last.""" 
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _case(B, Hq, Hkv, bs, seed):
    rng = np.random.default_rng(seed)
    lens = np.round(np.exp(rng.uniform(np.log(1), np.log(6000), B))).astype(np.int32)
    lens[0] = 0
    pages = (lens + bs - 1) // bs
    nb = int(pages.sum()) + 3
    width = int(pages.max()) + 1
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((B, width), -1, np.int32)
    used = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[used:used + pages[b]]
        used += pages[b]
    q = bf16(rng.standard_normal((B, Hq, 128)))
    cache = bf16(rng.standard_normal((2, nb, bs, Hkv, 128)))
    t = lambda x, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(x)).to(dt).cuda()
    oracle = oatt.decode_attention(q, cache[0], cache[1], bt, lens, 1.0 / math.sqrt(128))
    return t(q), t(cache), t(bt, torch.int32), t(lens, torch.int32), oracle


def _args(q, cache, bt, lens, out):
    B, Hq, D = q.shape
    k, v = cache[0], cache[1]
    nb, bs, Hkv, _ = k.shape
    return [q.data_ptr(), k.data_ptr(), v.data_ptr(), bt.data_ptr(), lens.data_ptr(),
            out.data_ptr(), B, Hq, Hkv, D, nb, bs, bt.shape[1], bt.stride(0),
            k.stride(0), k.stride(1), k.stride(2), 1.0 / math.sqrt(D)]


@pytest.mark.parametrize("B,Hq,Hkv,bs", [(64, 32, 8, 16), (7, 64, 8, 32), (300, 4, 1, 16)])
def test_noalloc_matches_workspace_decode_twice(B, Hq, Hkv, bs):
    from vllm_b200 import _native
    lib = _native.load()
    q, cache, bt, lens, oracle = _case(B, Hq, Hkv, bs, seed=B + Hq)
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty_like(q)
    ws_bytes = lib.vj_paged_decode_workspace_size(B, Hq, 128, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _native.check(lib.vj_paged_decode(*_args(q, cache, bt, lens, ref), 0, ws.data_ptr(),
                                      ws_bytes, stream))
    outs = []
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _native.check(lib.vj_paged_decode_noalloc(*_args(q, cache, bt, lens, out), stream))
        outs.append(out)
    torch.cuda.synchronize()
    r = ref.float().cpu().numpy()
    for out in outs:
        o = out.float().cpu().numpy()
        assert np.isfinite(o).all()
        for want in (r, oracle):
            err = np.abs(o - want)
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
    assert np.all(outs[0].float().cpu().numpy()[0] == 0)   # length-0 sequence


def test_noalloc_rejects_shapes_beyond_fixed_scratch():
    from vllm_b200 import _native
    lib = _native.load()
    cap = lib.vj_paged_decode_noalloc_scratch_bytes()
    assert cap == 16 << 20
    B = 1008                                   # first batch that does not fit at Hq = 32
    q = torch.zeros((B, 32, 128), dtype=torch.bfloat16, device="cuda")
    cache = torch.zeros((2, 4, 16, 8, 128), dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros((B, 1), dtype=torch.int32, device="cuda")
    lens = torch.ones(B, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    st = lib.vj_paged_decode_noalloc(*_args(q, cache, bt, lens, out),
                                     torch.cuda.current_stream().cuda_stream)
    assert st == _native.VJ_ERR_UNSUPPORTED
    assert b"fixed scratch" in lib.vj_get_last_error()
    # one sequence fewer fits
    st = lib.vj_paged_decode_noalloc(*_args(q[:1007], cache, bt[:1007], lens[:1007], out),
                                     torch.cuda.current_stream().cuda_stream)
    assert st == _native.VJ_OK
    torch.cuda.synchronize()
