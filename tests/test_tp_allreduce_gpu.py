"""Fused all-reduce + residual add + RMSNorm (vj_allreduce_add_rmsnorm) on
ONE GPU: the ranks' communication regions all live on this device and the
flags a CTA waits on are pre-set, so a single launch runs with nothing to
wait for (kernels that wait on one another never run as separate launches on
one GPU). Checks the arithmetic bit for bit: fp32 sum of the partials in rank
order, rounded to bf16, then exactly vj_add_rmsnorm; every rank's result is
identical. The cross-GPU path is covered by test_tp_nvlink_gpu.py."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _region(lib, world, rows, hidden):
    from vllm_b200 import _native
    flag_bytes = int(lib.vj_tp_flags_bytes(world))
    buf_bytes = (rows * hidden * 2 + 4095) // 4096 * 4096
    p = ctypes.c_void_p()
    _native.check(lib.vj_comm_alloc(flag_bytes + 2 * buf_bytes, ctypes.byref(p)))
    return p.value, flag_bytes, buf_bytes


@pytest.mark.parametrize("world,rows,hidden", [(1, 7, 1024), (2, 64, 4096), (4, 33, 5120),
                                               (8, 5, 2048)])
def test_fused_allreduce_matches_sum_then_add_rmsnorm(world, rows, hidden):
    from vllm_b200 import _native
    from vllm_b200.kernels.fused import add_rmsnorm
    from vllm_b200.src.tp_comm import device_view
    lib = _native.load()
    dev = torch.device("cuda", 0)
    G = int(lib.vj_tp_grid())
    regions = [_region(lib, world, rows, hidden) for _ in range(world)]
    g = torch.Generator(device="cpu").manual_seed(world * 100 + rows)
    parts = [torch.randn(rows, hidden, generator=g).bfloat16().to(dev) for _ in range(world)]
    x = torch.randn(rows, hidden, generator=g).bfloat16().to(dev)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).bfloat16().to(dev)
    site = 1
    for (base, fb, bb), pt in zip(regions, parts):
        device_view(base + fb + site * bb, (rows, hidden), torch.bfloat16, dev).copy_(pt)
        # flags this rank waits on: already far past any epoch
        device_view(base, (2 * world * G,), torch.int32, dev).fill_(1 << 30)
    s = torch.zeros(rows, hidden, dtype=torch.float32, device=dev)
    for pt in parts:
        s += pt.float()
    ref_x, ref_y = add_rmsnorm(s.bfloat16(), w, 1e-6, residual=x)
    bufs = (ctypes.c_void_p * world)(*[b + fb + site * bb for b, fb, bb in regions])
    flags = (ctypes.c_void_p * world)(*[b for b, _, _ in regions])
    for rank in range(world):
        x_out = torch.empty_like(x)
        y = torch.empty_like(x)
        _native.call("vj_allreduce_add_rmsnorm", ctypes.cast(bufs, ctypes.c_void_p), None,
                     ctypes.cast(flags, ctypes.c_void_p), ctypes.c_void_p(regions[rank][0]),
                     rank, world, x.data_ptr(), w.data_ptr(), x_out.data_ptr(), y.data_ptr(),
                     rows, hidden, 1e-6, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        err = device_view(regions[rank][0] + (2 * world + 1) * G * 4, (1,), torch.int32, dev)
        assert int(err.item()) == 0
        assert torch.equal(x_out, ref_x), f"rank {rank}: residual differs"
        assert torch.equal(y, ref_y), f"rank {rank}: normed output differs"
    for base, _, _ in regions:
        _native.check(lib.vj_comm_free(ctypes.c_void_p(base)))


@pytest.mark.parametrize("world,rows,hidden", [(4, 65, 4096), (8, 300, 5120), (8, 64, 1024),
                                               (4, 1000, 4096)])
def test_fused_allreduce_two_shot_arithmetic(world, rows, hidden):
    """Two-shot path (result buffers, more than 64 rows): rank r reduces its
    slice of rows into its result buffer and gathers the other slices from the
    peers' result buffers. On one GPU with pre-set flags every rank launches
    in turn; the first round computes every slice, the second gathers them."""
    from vllm_b200 import _native
    from vllm_b200.kernels.fused import add_rmsnorm
    from vllm_b200.src.tp_comm import device_view
    lib = _native.load()
    dev = torch.device("cuda", 0)
    G = int(lib.vj_tp_grid())
    flag_bytes = int(lib.vj_tp_flags_bytes(world))
    bb = (rows * hidden * 2 + 4095) // 4096 * 4096
    regions = []
    for _ in range(world):
        p = ctypes.c_void_p()
        _native.check(lib.vj_comm_alloc(flag_bytes + 4 * bb, ctypes.byref(p)))
        regions.append(p.value)
    g = torch.Generator(device="cpu").manual_seed(world * 1000 + rows)
    parts = [torch.randn(rows, hidden, generator=g).bfloat16().to(dev) for _ in range(world)]
    x = torch.randn(rows, hidden, generator=g).bfloat16().to(dev)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).bfloat16().to(dev)
    site = 0
    for base, pt in zip(regions, parts):
        device_view(base + flag_bytes + site * bb, (rows, hidden), torch.bfloat16, dev).copy_(pt)
        device_view(base, (2 * world * G,), torch.int32, dev).fill_(1 << 30)
    s = torch.zeros(rows, hidden, dtype=torch.float32, device=dev)
    for pt in parts:
        s += pt.float()
    ref_x, ref_y = add_rmsnorm(s.bfloat16(), w, 1e-6, residual=x)
    bufs = (ctypes.c_void_p * world)(*[b + flag_bytes + site * bb for b in regions])
    results = (ctypes.c_void_p * world)(*[b + flag_bytes + (2 + site) * bb for b in regions])
    flags = (ctypes.c_void_p * world)(*regions)
    outs = {}
    for rnd in range(2):
        # each launch stores its epoch into the other regions' flags: re-arm
        # them so that no launch of this round waits
        torch.cuda.synchronize()
        for base in regions:
            device_view(base, (2 * world * G,), torch.int32, dev).fill_(1 << 30)
        for rank in range(world):
            x_out, y = torch.empty_like(x), torch.empty_like(x)
            _native.call("vj_allreduce_add_rmsnorm", ctypes.cast(bufs, ctypes.c_void_p),
                         ctypes.cast(results, ctypes.c_void_p),
                         ctypes.cast(flags, ctypes.c_void_p), ctypes.c_void_p(regions[rank]),
                         rank, world, x.data_ptr(), w.data_ptr(), x_out.data_ptr(),
                         y.data_ptr(), rows, hidden, 1e-6,
                         torch.cuda.current_stream().cuda_stream)
            outs[rank] = (x_out, y)
        torch.cuda.synchronize()
    for rank in range(world):
        err = device_view(regions[rank] + (2 * world + 1) * G * 4, (1,), torch.int32, dev)
        assert int(err.item()) == 0
        x_out, y = outs[rank]
        assert torch.equal(x_out, ref_x), f"rank {rank}: residual differs"
        assert torch.equal(y, ref_y), f"rank {rank}: normed output differs"
    for base in regions:
        _native.check(lib.vj_comm_free(ctypes.c_void_p(base)))


def test_fused_allreduce_rejects_bad_arguments():
    from vllm_b200 import _native
    lib = _native.load()
    null = (ctypes.c_void_p * 2)(None, None)
    st = lib.vj_allreduce_add_rmsnorm(ctypes.cast(null, ctypes.c_void_p), None,
                                      ctypes.cast(null, ctypes.c_void_p), None, 0, 9, None,
                                      None, None, None, 4, 1024, 1e-6, None)
    assert st == _native.VJ_ERR_INVALID_ARGUMENT
    st = lib.vj_allreduce_add_rmsnorm(ctypes.cast(null, ctypes.c_void_p), None,
                                      ctypes.cast(null, ctypes.c_void_p), None, 0, 2, None,
                                      None, None, None, 4, 10000, 1e-6, None)
    assert st == _native.VJ_ERR_UNSUPPORTED


def test_peer_wait_times_out_into_the_error_word():
    """A peer that never announces: every CTA's wait gives up after its bound
    (2 s), sets the error word and returns; the context stays usable. One
    launch on one GPU with a flag nothing sets -- no second kernel waits on it."""
    import time

    from vllm_b200 import _native
    from vllm_b200.kernels.fused import add_rmsnorm
    from vllm_b200.src.tp_comm import device_view
    lib = _native.load()
    dev = torch.device("cuda", 0)
    G = int(lib.vj_tp_grid())
    world, rows, hidden = 2, 4, 1024
    regions = [_region(lib, world, rows, hidden) for _ in range(world)]
    bufs = (ctypes.c_void_p * world)(*[b + fb for b, fb, _ in regions])
    flags = (ctypes.c_void_p * world)(*[b for b, _, _ in regions])
    x = torch.ones(rows, hidden, dtype=torch.bfloat16, device=dev)
    w = torch.ones(hidden, dtype=torch.bfloat16, device=dev)
    xo, y = torch.empty_like(x), torch.empty_like(x)
    t0 = time.perf_counter()
    _native.call("vj_allreduce_add_rmsnorm", ctypes.cast(bufs, ctypes.c_void_p), None,
                 ctypes.cast(flags, ctypes.c_void_p), ctypes.c_void_p(regions[0][0]), 0, world,
                 x.data_ptr(), w.data_ptr(), xo.data_ptr(), y.data_ptr(), rows, hidden, 1e-6,
                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    err = device_view(regions[0][0] + (2 * world + 1) * G * 4, (1,), torch.int32, dev)
    assert int(err.item()) == 1
    assert 1.5 < waited < 30
    # the device still works
    r, h = add_rmsnorm(x, w, 1e-6, residual=x)
    torch.cuda.synchronize()
    assert torch.isfinite(h.float()).all()
    for base, _, _ in regions:
        _native.check(lib.vj_comm_free(ctypes.c_void_p(base)))
