"""Generate host-side golden traces by running the reference's OWN Python code.

Imports, from the vllm-jax checkout named by $VLLM_JAX_REF (or the first
command-line argument):
  vllm/src/request.py, vllm/src/kv_cache_manager.py, vllm/src/scheduler.py,
  vllm/config.py, vllm/sampling_params.py      -- unmodified, pure Python
  vllm/src/model_runner.py                      -- its prepare_prefill /
      prepare_decode / pad_block_tables / _bucket_size, with jax/flax/
      transformers replaced by import stubs (jax.numpy -> numpy; the jitted
      model steps are never called)
and drives them with the loop of vllm/src/engine.py:44-75 (Engine.step /
generate), feeding a deterministic stand-in for the sampled token. Every
scheduled step's decode/prefill request ids and the packed batch arrays are
written to tests/golden/host_traces.json.

The reference cannot be imported under its own package name here (an
unrelated `vllm` distribution is installed), so its modules are loaded from
their files into a private `vllm` namespace inside this process only.

Run:  VLLM_JAX_REF=<vllm-jax checkout> python tests/golden/make_golden.py
"""
from __future__ import annotations

import dataclasses
import importlib.util
import itertools
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VLLM_JAX_REF", "."))
OUT = Path(__file__).resolve().parent / "host_traces.json"


def _stub_modules():
    """Minimal stand-ins so model_runner.py imports; none of them computes."""
    jax = types.ModuleType("jax")
    jax.numpy = np
    jax.Array = np.ndarray
    jax.devices = lambda *a: ["cpu"]
    jax.device_put = lambda x, device=None: x
    jax.random = types.SimpleNamespace(PRNGKey=lambda s: s)
    exp = types.ModuleType("jax.experimental")
    exp.mesh_utils = types.SimpleNamespace(create_device_mesh=lambda *a, **k: None)
    sharding = types.ModuleType("jax.sharding")
    sharding.Mesh = lambda *a, **k: None
    sharding.set_mesh = lambda *a, **k: None
    flax = types.ModuleType("flax")
    nnx = types.SimpleNamespace(jit=lambda f: f, Module=object)
    struct = types.SimpleNamespace(
        dataclass=dataclasses.dataclass,
        field=lambda pytree_node=True, **kw: dataclasses.field(**kw))
    flax.nnx, flax.struct = nnx, struct
    transformers = types.ModuleType("transformers")
    transformers.Qwen3Config = object
    qwen3 = types.ModuleType("vllm.model.qwen3")
    qwen3.DecodeAttentionMetadata = qwen3.PrefillAttentionMetadata = object
    qwen3.Qwen3ForCausalLM = object
    sampler = types.ModuleType("vllm.sampler")
    sampler.Sampler = object
    hf = types.ModuleType("vllm.utils.hf_convert")
    hf.load_hf_weights_into_model = lambda *a, **k: None
    for name, mod in {"jax": jax, "jax.numpy": np, "jax.experimental": exp,
                      "jax.experimental.mesh_utils": exp.mesh_utils,
                      "jax.sharding": sharding, "flax": flax, "transformers": transformers,
                      "vllm.model": types.ModuleType("vllm.model"), "vllm.model.qwen3": qwen3,
                      "vllm.sampler": sampler, "vllm.utils": types.ModuleType("vllm.utils"),
                      "vllm.utils.hf_convert": hf}.items():
        sys.modules[name] = mod


def _load(name: str, rel: str):
    spec = importlib.util.spec_from_file_location(name, REF / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_reference():
    for name in ("vllm", "vllm.src"):
        pkg = types.ModuleType(name)
        pkg.__path__ = []
        sys.modules[name] = pkg
    _stub_modules()
    ref = types.SimpleNamespace()
    ref.config = _load("vllm.config", "vllm/config.py")
    ref.sampling_params = _load("vllm.sampling_params", "vllm/sampling_params.py")
    ref.request = _load("vllm.src.request", "vllm/src/request.py")
    ref.kv = _load("vllm.src.kv_cache_manager", "vllm/src/kv_cache_manager.py")
    ref.scheduler = _load("vllm.src.scheduler", "vllm/src/scheduler.py")
    ref.model_runner = _load("vllm.src.model_runner", "vllm/src/model_runner.py")
    return ref


def fake_token(req_id: int, n_completion: int, vocab: int) -> int:
    """Deterministic stand-in for the sampled token (model numerics excluded)."""
    return (req_id * 7919 + n_completion * 104729 + 13) % vocab


def _arr(x):
    return np.asarray(x).tolist()


def run_scenario(ref, name, cfg_kw, prompt_lens, sp_kw, eos_token_id=151645, vocab=151936,
                 eos_at=None, seed=0, max_steps=10_000):
    ref.request.Request.counter = itertools.count()      # ids start at 0 per scenario
    cfg = ref.config.Config(model="synthetic", **cfg_kw)
    kvm = ref.kv.KVCacheManager(cfg.num_blocks, cfg.block_size)
    sched = ref.scheduler.Scheduler(cfg, kvm)
    runner = object.__new__(ref.model_runner.ModelRunner)
    runner.block_size = cfg.block_size
    runner.max_num_batched_tokens = cfg.max_num_batched_tokens
    runner.max_num_seqs = cfg.max_num_seqs
    runner.max_blocks_per_seq = (cfg.max_num_batched_tokens + cfg.block_size - 1) // cfg.block_size
    runner.kv_cache_manager = kvm
    runner._to_device = lambda v: v
    sp = ref.sampling_params.SamplingParams(**sp_kw)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, vocab, size=n).tolist() for n in prompt_lens]
    reqs = [ref.request.Request(token_ids=p, sampling_params=sp, eos_token_id=eos_token_id)
            for p in prompts]
    for r in reqs:
        sched.add(r)
    steps = []
    outcome = "finished"
    while not sched.is_finished():
        if len(steps) >= max_steps:
            outcome = "step_cap"
            break
        try:
            dec, pre = sched.schedule()
        except AssertionError as e:   # scheduler.py:37 "Request cant fit in memory"
            outcome = f"assert: {e}"
            break
        rec = {"decode_ids": [r.id for r in dec], "prefill_ids": [r.id for r in pre],
               "waiting_ids": [r.id for r in sched.waiting],
               "running_ids": [r.id for r in sched.running]}
        tokens = []
        if dec:
            b = runner.prepare_decode(dec)
            rec["decode"] = {"input_ids": _arr(b.input_ids), "positions": _arr(b.positions),
                             "slot_mapping": _arr(b.slot_mapping),
                             "block_tables": _arr(b.block_tables),
                             "context_lens": _arr(b.context_lens)}
            for r in dec:
                t = fake_token(r.id, r.num_completion_tokens, vocab)
                if eos_at is not None and (r.id, r.num_completion_tokens) in eos_at:
                    t = eos_token_id
                r.token_ids.append(t)
                r.num_completion_tokens += 1
                tokens.append(t)
        if pre:
            b = runner.prepare_prefill(pre)
            rec["prefill"] = {"input_ids": _arr(b.input_ids), "positions": _arr(b.positions),
                              "slot_mapping": _arr(b.slot_mapping),
                              "block_tables": _arr(b.block_tables),
                              "cu_seqlens_q": _arr(b.cu_seqlens_q),
                              "cu_seqlens_k": _arr(b.cu_seqlens_k),
                              "max_seqlen_q": int(b.max_seqlen_q),
                              "max_seqlen_k": int(b.max_seqlen_k),
                              "max_seqlen_bucket": int(b.max_seqlen_bucket)}
        sched.postprocess(dec, tokens)
        rec["sampled"] = tokens
        rec["finished"] = [r.id for r in dec if r.is_finished()]
        rec["free_blocks"] = [blk.block_id for blk in kvm.free_block_queue]
        steps.append(rec)
    return {"name": name, "config": cfg_kw, "prompt_lens": list(prompt_lens),
            "sampling": sp_kw, "eos_token_id": eos_token_id, "vocab": vocab, "seed": seed,
            "eos_at": sorted(list(eos_at)) if eos_at else [],
            "prompts": prompts, "steps": steps, "outcome": outcome, "max_steps": max_steps,
            "final_tokens": {r.id: r.token_ids for r in reqs}}


SCENARIOS = [
    # C1: the tiny end-to-end config (prompts 17/64/129/300, 32 greedy tokens)
    dict(name="c1", cfg_kw=dict(max_num_batched_tokens=512, max_num_seqs=4, num_blocks=128,
                                block_size=16),
         prompt_lens=[17, 64, 129, 300],
         sp_kw=dict(temperature=0.0, max_new_tokens=32, ignore_eos=True)),
    # the reference smoke config (test.py:10-16) with more prompts than seats
    dict(name="smoke_cfg_many", cfg_kw=dict(max_num_batched_tokens=128, max_num_seqs=4,
                                            num_blocks=128, block_size=16),
         prompt_lens=[5, 9, 30, 17, 40, 3, 60, 12],
         sp_kw=dict(temperature=0.0, max_new_tokens=16, ignore_eos=True)),
    # pool pressure: decode-time block allocation preempts the tail; finished
    # requests never return their blocks (scheduler.py:65-70), so the run then
    # ends in the reference's assert (scheduler.py:37) ...
    dict(name="preempt_assert", cfg_kw=dict(max_num_batched_tokens=256, max_num_seqs=3,
                                            num_blocks=10, block_size=16),
         prompt_lens=[47, 52, 12, 33, 48],
         sp_kw=dict(temperature=0.0, max_new_tokens=47, ignore_eos=True)),
    # ... or the victim is never re-admitted (recorded up to a step cap)
    dict(name="preempt_stall", cfg_kw=dict(max_num_batched_tokens=256, max_num_seqs=3,
                                           num_blocks=14, block_size=16),
         prompt_lens=[16, 21, 50, 35],
         sp_kw=dict(temperature=0.0, max_new_tokens=50, ignore_eos=True), max_steps=120),
    # EOS finishes some requests early (not ignored)
    dict(name="eos", cfg_kw=dict(max_num_batched_tokens=256, max_num_seqs=3, num_blocks=64,
                                 block_size=16),
         prompt_lens=[10, 50, 16, 33, 7],
         sp_kw=dict(temperature=0.0, max_new_tokens=20, ignore_eos=False),
         eos_at={(1, 3), (0, 10), (3, 0)}),
    # block_size 32 and a budget boundary (num_batched + len >= budget is refused)
    dict(name="bs32_budget", cfg_kw=dict(max_num_batched_tokens=100, max_num_seqs=8,
                                         num_blocks=40, block_size=32),
         prompt_lens=[40, 59, 60, 1, 99, 33],
         sp_kw=dict(temperature=0.0, max_new_tokens=9, ignore_eos=True)),
]


def main():
    ref = load_reference()
    out = [run_scenario(ref, **sc) for sc in SCENARIOS]
    with open(OUT, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {sum(len(s['steps']) for s in out)} steps)")


if __name__ == "__main__":
    main()
