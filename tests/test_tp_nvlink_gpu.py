"""Tensor parallelism over NVLink on 2 GPUs (skipped with fewer).

Two processes (one per GPU, NCCL for setup only) build a TPComm (one-shot,
then two-shot) and run the fused all-reduce + add + RMSNorm many times,
alternating the two buffers, in eager mode and replayed from a CUDA graph;
every result must equal, bit for
bit, the fp32 rank-order sum of the partials (gathered with NCCL) followed
by vj_add_rmsnorm. Then a 2-rank Engine with the NVLink path generates with
CUDA-graph decode and must agree with the NCCL path on the first tokens.
Every wait is bounded: the process group has a short timeout and the
parent kills its own children if they do not report back.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check_comm(comm, rank, world, dev, H):
    import torch.distributed as dist

    from vllm_b200.kernels.fused import add_rmsnorm
    g = torch.Generator(device="cpu").manual_seed(1234)
    w = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16().to(dev)

    def reference(part, x):
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        s = torch.zeros(part.shape, dtype=torch.float32, device=dev)
        for p in parts:
            s += p.float()
        return add_rmsnorm(s.bfloat16(), w, 1e-6, residual=x)

    gl = torch.Generator(device="cpu").manual_seed(77 + rank)
    for it in range(24):
        T = [1, 7, 64, 96][it % 4]
        site = it % 2
        part = torch.randn(T, H, generator=gl).bfloat16().to(dev)
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(it)).bfloat16().to(dev)
        comm.buffer(site, T).copy_(part)
        xo, y = comm.allreduce_add_rmsnorm(site, T, x, w, 1e-6)
        rx, ry = reference(part, x)
        assert torch.equal(xo, rx) and torch.equal(y, ry), f"eager call {it} differs"
    # CUDA graph of four calls (both buffers twice), replayed with new inputs
    T = 32
    src = [torch.zeros(T, H, dtype=torch.bfloat16, device=dev) for _ in range(4)]
    xin = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            cur = xin
            outs = []
            for k in range(4):
                comm.buffer(k % 2, T).copy_(src[k])
                cur, y = comm.allreduce_add_rmsnorm(k % 2, T, cur, w, 1e-6)
                outs.append((cur, y))
    torch.cuda.current_stream(dev).wait_stream(s)
    for rep in range(3):
        for k in range(4):
            src[k].copy_(torch.randn(T, H, generator=gl).bfloat16())
        xin.copy_(torch.randn(T, H, generator=torch.Generator().manual_seed(900 + rep))
                  .bfloat16())
        graph.replay()
        torch.cuda.synchronize(dev)
        cur = xin.clone()
        for k in range(4):
            rx, ry = reference(src[k], cur)
            assert torch.equal(outs[k][0], rx) and torch.equal(outs[k][1], ry), \
                f"graph replay {rep} call {k} differs"
            cur = rx
    assert not comm.failed()
    del graph
    comm.close()


def _worker(rank, world, port, q, engine_check=True):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "vllm-jax_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from vllm_b200.src.tp_comm import TPComm
        H, R = 2048, 96
        for two_shot in (False, True):
            _check_comm(TPComm(dist.group.WORLD, rank, world, dev, R, H, two_shot=two_shot),
                        rank, world, dev, H)
        if not engine_check:
            q.put((rank, "ok"))
            return
        # engine: NVLink path (CUDA-graph decode) vs NCCL path (eager)
        from vllm_b200 import Config, SamplingParams
        from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
        from vllm_b200.src.engine import Engine
        from vllm_b200.src.request import Request
        cfg = Qwen3Config(vocab_size=4096, hidden_size=512, intermediate_size=1024,
                          num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=4)
        wts = Qwen3Weights(cfg, dev, seed=5, tp_rank=rank, tp_size=world)
        prompts = [[(7 * i + 3 * j) % 4096 for j in range(n)] for i, n in enumerate((30, 70, 9))]
        res = {}
        for mode in ("nvlink", "nccl"):
            Request.reset_ids()
            eng = Engine(Config(model="tiny", max_num_batched_tokens=256, max_num_seqs=4,
                                num_blocks=64, block_size=16, compat=False,
                                tensor_parallel_size=world, tp_allreduce=mode), dev,
                         model_config=cfg, weights=wts, max_slots=8,
                         process_group=dist.group.WORLD)
            assert eng.runner.use_cuda_graphs == (mode == "nvlink")
            res[mode] = eng.generate(prompts, SamplingParams(temperature=0, max_new_tokens=8,
                                                             ignore_eos=True))
            eng.close()
        assert [o[:2] for o in res["nvlink"]] == [o[:2] for o in res["nccl"]], res
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent, never hang it
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()[-1500:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, engine_check):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, engine_check))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, msg = q.get(timeout=420)
            results[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results == {r: "ok" for r in range(world)}, results


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nvlink_fused_allreduce_two_ranks():
    _run(2, True)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_nvlink_fused_allreduce_all_ranks():
    """Every GPU of the box (4 or 8 ranks), one-shot and two-shot."""
    n = torch.cuda.device_count()
    _run(8 if n >= 8 else 4, False)
