"""Continuous-batching engine with vllm-jax's API (vllm/src/engine.py:13-75).

`Engine(config).generate(prompts, **sampling_kwargs)` runs the reference's
loop: schedule -> model step -> postprocess until every request finished.
Prompts may be token-id lists (no tokenizer is needed) or strings, which
require a `tokenizer` object with encode/decode (HF weights and tokenizers
are not downloadable here, so the model is the random-init architecture the
benchmarks name). `LLM` is an alias: the reference has no class of that name
and north_star's LLM.generate maps to Engine.generate.

Tensor parallelism: launch one process per GPU (torchrun) with
config.tensor_parallel_size = world size; every rank runs the same
deterministic scheduler on the same requests, so the batches agree and no
host broadcast is needed; the model all-reduces after o_proj and down_proj.
"""
from __future__ import annotations

import dataclasses
import os
import time

import torch

from ..config import Config
from ..model.qwen3 import Qwen3Config, Qwen3Weights, get_config
from ..sampling_params import SamplingParams
from .kv_cache_manager import KVCacheManager
from .model_runner import ModelRunner, kv_cache_bytes_per_block
from .request import Request
from .scheduler import ChunkedScheduler, Scheduler


class Engine:

    def __init__(self, config: Config, device: torch.device | None = None, *,
                 model_config: Qwen3Config | None = None, tokenizer=None, seed: int = 0,
                 eos_token_id: int | None = 151645, process_group=None,
                 weights: Qwen3Weights | None = None, max_slots: int = 4096,
                 use_cuda_graphs: bool = True):
        self.config = config
        self.tokenizer = tokenizer
        self.eos_token_id = (tokenizer.eos_token_id if tokenizer is not None
                             else eos_token_id)
        self.tp_size = config.tensor_parallel_size
        self.tp_rank = 0
        if self.tp_size > 1:
            if not torch.distributed.is_initialized():
                raise RuntimeError("tensor_parallel_size > 1 needs torch.distributed "
                                   "initialised (one process per GPU)")
            self.tp_rank = torch.distributed.get_rank(process_group)
            if torch.distributed.get_world_size(process_group) != self.tp_size:
                raise ValueError("tensor_parallel_size must equal the process group size")
        if device is None:
            device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
        self.device = device
        # config.model: a preset name (random-init weights of that architecture)
        # or a local Hugging Face checkpoint directory (weights loaded, sharded)
        hf_dir = config.model if os.path.isdir(config.model) else None
        if model_config is not None:
            self.mcfg = model_config
        elif hf_dir:
            from ..model.hf_loader import config_from_hf
            self.mcfg = config_from_hf(hf_dir)
        else:
            self.mcfg = get_config(config.model)
        if weights is None and hf_dir:
            from ..model.hf_loader import load_hf_weights
            weights = load_hf_weights(hf_dir, device, self.tp_rank, self.tp_size, self.mcfg)
        if tokenizer is None and hf_dir and os.path.exists(
                os.path.join(hf_dir, "tokenizer_config.json")):
            from transformers import AutoTokenizer
            self.tokenizer = tokenizer = AutoTokenizer.from_pretrained(hf_dir,
                                                                       local_files_only=True)
            self.eos_token_id = tokenizer.eos_token_id
        self.weights = weights or Qwen3Weights(self.mcfg, device, seed, self.tp_rank,
                                               self.tp_size)
        if config.fused_gemm_max_rows > 0:
            # packed copies of the projection weights, before the pool is sized
            self.weights.pack_tiles()
        num_blocks = config.num_blocks
        if num_blocks <= 0:
            free, _ = torch.cuda.mem_get_info(device)
            per = kv_cache_bytes_per_block(self.mcfg, config.block_size, self.tp_size)
            num_blocks = int(free * config.gpu_memory_utilization) // per
            if self.tp_size > 1:   # every rank must agree on the pool size
                t = torch.tensor([num_blocks], device=device)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN,
                                             group=process_group)
                num_blocks = int(t.item())
            self.config = config = dataclasses.replace(config, num_blocks=num_blocks)
        if config.enable_prefix_caching and not config.enable_chunked_prefill:
            raise ValueError("enable_prefix_caching needs enable_chunked_prefill")
        if config.enable_chunked_prefill:
            if config.compat:
                self.config = config = dataclasses.replace(config, compat=False)
            if num_blocks < config.max_blocks_per_seq:
                raise ValueError("chunked prefill needs a pool of at least max_model_len tokens")
        self.tp_comm = None
        if self.tp_size > 1 and config.tp_allreduce == "nvlink":
            from ..kernels.metadata import bucket_size
            from .tp_comm import TPComm
            self.tp_comm = TPComm(process_group or torch.distributed.group.WORLD, self.tp_rank,
                                  self.tp_size, device,
                                  max(1024, bucket_size(max(config.max_num_seqs, 1))),
                                  self.mcfg.hidden_size)
        elif config.tp_allreduce not in ("nvlink", "nccl"):
            raise ValueError("tp_allreduce must be 'nvlink' or 'nccl'")
        self.kv = KVCacheManager(num_blocks, config.block_size)
        self.scheduler = (ChunkedScheduler(config, self.kv) if config.enable_chunked_prefill
                          else Scheduler(config, self.kv))
        self.trace: list | None = None     # set to a list to record chunked steps
        self.runner = ModelRunner(config, self.mcfg, self.kv, device, tp_rank=self.tp_rank,
                                  tp_size=self.tp_size, process_group=process_group,
                                  weights=self.weights, max_slots=max_slots,
                                  use_cuda_graphs=use_cuda_graphs, tp_comm=self.tp_comm)
        self.live: dict[int, Request] = {}
        self.stats = {"steps": 0, "decode_tokens": 0, "prefill_tokens": 0, "decode_steps": 0,
                      "decode_s": 0.0, "prefill_s": 0.0, "decode_ctx_tokens": 0,
                      "h2d_bytes": 0, "d2h_bytes": 0}

    def close(self) -> None:
        """Release the decode CUDA graphs and, under tensor parallelism, the
        NVLink communicator (collective: every rank calls it). Call before
        torch.distributed.destroy_process_group."""
        self.runner.graphs.clear()
        if self.tp_comm is not None:
            self.tp_comm.close()
            self.tp_comm = None
            self.runner.model.tp_comm = None

    # ---------------------------------------------------------------- requests
    def preprocess(self, prompt) -> list[int]:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("string prompts need a tokenizer; pass token-id lists")
            return list(self.tokenizer.encode(prompt))
        return [int(t) for t in prompt]

    def add_request(self, request: Request) -> None:
        if len(request) + request.max_new_tokens > self.config.max_len:
            raise ValueError(f"request {request.id}: {len(request)} prompt + "
                             f"{request.max_new_tokens} new tokens exceed max_model_len "
                             f"{self.config.max_len}")
        self.live[request.id] = request
        self.scheduler.add(request)

    # ---------------------------------------------------------------- loop
    def step(self) -> list[tuple[int, int]]:
        if self.config.enable_chunked_prefill:
            return self._step_chunked()
        decode, prefill = self.scheduler.schedule()
        st = self.stats
        st["decode_ctx_tokens"] += sum(len(r) for r in decode)
        tokens = self.runner.run(decode, prefill, self.live, st)
        self.scheduler.postprocess(decode, tokens)
        st["steps"] += 1
        st["decode_tokens"] += len(decode)
        st["decode_steps"] += 1 if decode else 0
        st["prefill_tokens"] += sum(len(r) for r in prefill)
        done = []
        for r in decode:
            if r.is_finished():
                done.append((r.id, r.num_completion_tokens))
                self.runner.release(r)
                del self.live[r.id]
        return done

    def _step_chunked(self) -> list[tuple[int, int]]:
        batch = self.scheduler.schedule()
        if not batch:
            raise RuntimeError("chunked scheduler made no progress (pool too small?)")
        st = self.stats
        all_decode = all(n == 1 and r.num_computed_tokens + 1 == len(r) for r, n in batch)
        if all_decode:
            st["decode_ctx_tokens"] += sum(len(r) for r, _ in batch)
        if self.trace is not None:
            self.trace.append({"batch": [(r.id, r.num_computed_tokens, n) for r, n in batch],
                               "blocks": {r.id: self.kv.block_ids(r) for r, _ in batch}})
        sampled = self.runner.run_chunked(batch, self.live, st)
        self.scheduler.postprocess(batch, sampled)
        st["steps"] += 1
        st["decode_tokens"] += len(sampled)
        st["decode_steps"] += 1 if all_decode else 0
        st["prefill_tokens"] += sum(n for r, n in batch if n > 1 or r.id not in sampled)
        done = []
        for r, _ in batch:
            if r.is_finished():
                done.append((r.id, r.num_completion_tokens))
                self.runner.release(r)
                del self.live[r.id]
        return done

    # ---------------------------------------------------------------- async loop
    @property
    def async_scheduling(self) -> bool:
        c = self.config
        return c.async_scheduling and not c.compat and not c.enable_chunked_prefill

    def _finish(self, r: Request) -> None:
        """Scheduler.postprocess's finish (compat=False: blocks released)."""
        from .request import Status
        r.status = Status.FINISHED
        sched = self.scheduler
        if r in sched.running:
            sched.running.remove(r)
        elif r in sched.waiting:              # preempted before its EOS was read
            sched.waiting.remove(r)
        sched.finished_requests.append(r)
        self.kv.deallocate(r)
        self.runner.release(r)
        self.live.pop(r.id, None)

    def _launch(self):
        """Schedule and enqueue one step while the previous one still runs.
        Decode rows get a placeholder token at once (the real one is already
        on its way into the device token table, which the next step reads);
        a request that reaches max_new_tokens finishes now."""
        decode, prefill = self.scheduler.schedule()
        if not decode and not prefill:
            return None
        st = self.stats
        t0 = time.perf_counter()
        st["decode_ctx_tokens"] += sum(len(r) for r in decode)
        pending = self.runner.launch(decode, prefill, self.live, st)
        slots = []
        for r in decode:
            r.token_ids.append(-1)
            r.num_completion_tokens += 1
            slots.append(len(r.token_ids) - 1)
            if r.num_completion_tokens == r.max_new_tokens:
                self._finish(r)
        st["steps"] += 1
        st["decode_tokens"] += len(decode)
        st["decode_steps"] += 1 if decode else 0
        st["prefill_tokens"] += sum(len(r) for r in prefill)
        return decode, slots, pending, bool(prefill), t0

    def _complete(self, step) -> None:
        """Fill a step's placeholders; a request that sampled EOS finishes
        here, and the token a later step already computed for it is dropped."""
        decode, slots, pending, had_prefill, t0 = step
        if pending is not None:
            for r, i, t in zip(decode, slots, pending.collect()):
                if i >= len(r.token_ids):          # stopped at an earlier EOS
                    continue
                r.token_ids[i] = t
                if not r.ignore_eos and t == r.eos_token_id:
                    del r.token_ids[i + 1:]
                    r.num_completion_tokens = len(r.token_ids) - r.num_prompt_tokens
                    if not r.is_finished():
                        self._finish(r)
        # wall time partitioned between steps (launches overlap earlier steps)
        now = time.perf_counter()
        key = "prefill_s" if had_prefill else "decode_s"
        self.stats[key] += now - max(t0, self._last_done)
        self._last_done = now

    def _run_async(self) -> None:
        """generate()'s loop with one step of lookahead: step k+1 is scheduled
        and enqueued before step k's tokens are read back, so host scheduling
        overlaps the GPU. Only EOS needs step k's tokens; a request that hits
        it is computed one extra step whose token is discarded."""
        pending = None
        self._last_done = time.perf_counter()
        while True:
            nxt = None if self.scheduler.is_finished() else self._launch()
            if pending is not None:
                self._complete(pending)
            elif nxt is None:
                if self.scheduler.is_finished():
                    break
                raise RuntimeError("scheduler made no progress (pool too small?)")
            pending = nxt
            if pending is None and self.scheduler.is_finished():
                break

    def generate(self, prompts, sampling_params: SamplingParams | list | None = None,
                 **kwargs):
        """vllm/src/engine.py:45-75. Returns, per prompt, the completion text
        (with a tokenizer) or the list of completion token ids."""
        if sampling_params is None:
            names = {f.name for f in dataclasses.fields(SamplingParams)}
            sampling_params = SamplingParams(**{k: v for k, v in kwargs.items() if k in names})
        params = (sampling_params if isinstance(sampling_params, list)
                  else [sampling_params] * len(prompts))
        reqs = []
        for i, (p, sp) in enumerate(zip(prompts, params)):
            r = Request(self.preprocess(p), sp, self.eos_token_id)
            # sampled tokens depend on (seed, prompt index, position) only, not
            # on how requests were batched
            r.sample_stream = i
            reqs.append(r)
            self.add_request(r)
        if self.async_scheduling:
            self._run_async()
        else:
            while not self.scheduler.is_finished():
                self.step()
        if self.tp_comm is not None and self.tp_comm.failed():
            raise RuntimeError("tensor-parallel all-reduce timed out waiting for a peer rank")
        outs = []
        for r in reqs:
            comp = r.token_ids[r.num_prompt_tokens:]
            outs.append(self.tokenizer.decode(comp) if self.tokenizer is not None else comp)
        return outs


LLM = Engine
