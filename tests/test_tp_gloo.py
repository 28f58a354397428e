"""Tensor-parallel host logic on CPU with 2 gloo ranks.

* Qwen3Weights shards (KV-head split of q/k/v and o_proj, split MLP) are
  exact slices of the unsharded model, and the row-parallel products summed
  by all_reduce (the model's o_proj / down_proj) equal the unsharded GEMMs.
* Every rank runs the same deterministic scheduler on the same requests and
  reaches the same batches, so no per-step broadcast is needed.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "vllm-jax_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from vllm_b200.config import Config
        from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
        from vllm_b200.sampling_params import SamplingParams
        from vllm_b200.src.kv_cache_manager import KVCacheManager
        from vllm_b200.src.request import Request
        from vllm_b200.src.scheduler import Scheduler

        cfg = Qwen3Config(hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                          num_attention_heads=8, num_key_value_heads=4, vocab_size=50)
        cpu = torch.device("cpu")
        full = Qwen3Weights(cfg, cpu, seed=3)
        part = Qwen3Weights(cfg, cpu, seed=3, tp_rank=rank, tp_size=world)
        D = cfg.head_dim
        hq_l, hkv_l = cfg.num_attention_heads // world, cfg.num_key_value_heads // world
        i_l = cfg.intermediate_size // world
        for lf, lp in zip(full.layers, part.layers):
            Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
            q_full = lf.w_qkv[:Hq * D]
            k_full = lf.w_qkv[Hq * D:(Hq + Hkv) * D]
            assert torch.equal(lp.w_qkv[:hq_l * D], q_full[rank * hq_l * D:(rank + 1) * hq_l * D])
            assert torch.equal(lp.w_qkv[hq_l * D:(hq_l + hkv_l) * D],
                               k_full[rank * hkv_l * D:(rank + 1) * hkv_l * D])
            assert torch.equal(lp.w_gate_up[:i_l], lf.w_gate_up[rank * i_l:(rank + 1) * i_l])
            # row-parallel o_proj: sum over ranks of the local products
            x = torch.randn(5, Hq * D, generator=torch.Generator().manual_seed(9)).bfloat16()
            xs = x[:, rank * hq_l * D:(rank + 1) * hq_l * D].float()
            partial = xs @ lp.w_o.float().T
            dist.all_reduce(partial)
            ref = x.float() @ lf.w_o.float().T
            assert torch.allclose(partial, ref, rtol=1e-4, atol=1e-3)
        assert torch.equal(part.embed, full.embed)
        # identical scheduling on every rank
        Request.reset_ids()
        conf = Config(model="x", max_num_batched_tokens=128, max_num_seqs=3, num_blocks=20,
                      block_size=16, tensor_parallel_size=world)
        kv = KVCacheManager(conf.num_blocks, conf.block_size)
        sched = Scheduler(conf, kv)
        g = torch.Generator().manual_seed(5)
        for n in (30, 50, 7, 90, 12):
            sched.add(Request(torch.randint(0, 50, (n,), generator=g).tolist(),
                              SamplingParams(temperature=0, max_new_tokens=9, ignore_eos=True), 0))
        trace = []
        while not sched.is_finished():
            dec, pre = sched.schedule()
            for r in dec:
                r.token_ids.append(1)
                r.num_completion_tokens += 1
            sched.postprocess(dec, [1] * len(dec))
            trace.append(([r.id for r in dec], [r.id for r in pre],
                          [b.block_id for b in kv.free_block_queue]))
        gathered = [None] * world
        dist.all_gather_object(gathered, trace)
        assert all(t == gathered[0] for t in gathered)
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent, never hang it
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp2_gloo_sharding_and_scheduling():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, msg = q.get(timeout=300)
        results[rank] = msg
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
