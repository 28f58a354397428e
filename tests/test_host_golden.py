"""Host logic vs golden traces recorded from the reference's own code.

tests/golden/host_traces.json was produced by tests/golden/make_golden.py,
which ran vllm-jax's scheduler.py / kv_cache_manager.py / request.py and the
unmodified prepare_prefill / prepare_decode of model_runner.py. Here the same
workloads are replayed through this build's Scheduler / KVCacheManager and
the oracle's restatement of the packing; every scheduled id, free-block
queue and packed array must match exactly (bit-exact integer parity)."""
import json
import os

import numpy as np
import pytest

from oracle import host as ohost

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "host_traces.json")


def _load():
    with open(GOLDEN) as f:
        return json.load(f)


def fake_token(req_id, n_completion, vocab):
    # same deterministic stand-in for the sampled token as make_golden.py
    return (req_id * 7919 + n_completion * 104729 + 13) % vocab


def replay(sc, on_step=None):
    """Drive this build's host side through scenario `sc`; yields per-step records."""
    from vllm_b200.config import Config
    from vllm_b200.sampling_params import SamplingParams
    from vllm_b200.src.kv_cache_manager import KVCacheManager
    from vllm_b200.src.request import Request
    from vllm_b200.src.scheduler import Scheduler

    Request.reset_ids()
    cfg = Config(model="synthetic", **sc["config"])
    kvm = KVCacheManager(cfg.num_blocks, cfg.block_size)
    sched = Scheduler(cfg, kvm)
    sp = SamplingParams(**sc["sampling"])
    reqs = [Request(p, sp, sc["eos_token_id"]) for p in sc["prompts"]]
    for r in reqs:
        sched.add(r)
    eos_at = {tuple(x) for x in sc["eos_at"]}
    width = cfg.max_blocks_per_seq
    out = []
    outcome = "finished"
    while not sched.is_finished():
        if len(out) >= sc["max_steps"]:
            outcome = "step_cap"
            break
        try:
            dec, pre = sched.schedule()
        except AssertionError as e:
            outcome = f"assert: {e}"
            break
        rec = {"decode_ids": [r.id for r in dec], "prefill_ids": [r.id for r in pre],
               "waiting_ids": [r.id for r in sched.waiting],
               "running_ids": [r.id for r in sched.running]}
        if on_step is not None:
            on_step(rec, dec, pre, kvm, cfg)
        toks = []
        if dec:
            rec["decode"] = ohost.prepare_decode([r.token_ids for r in dec],
                                                 [kvm.block_ids(r) for r in dec],
                                                 cfg.block_size, width)
            for r in dec:
                t = fake_token(r.id, r.num_completion_tokens, sc["vocab"])
                if (r.id, r.num_completion_tokens) in eos_at:
                    t = sc["eos_token_id"]
                r.token_ids.append(t)
                r.num_completion_tokens += 1
                toks.append(t)
        if pre:
            rec["prefill"] = ohost.prepare_prefill([r.token_ids for r in pre],
                                                   [kvm.block_ids(r) for r in pre],
                                                   cfg.block_size, cfg.max_num_seqs, width)
        sched.postprocess(dec, toks)
        rec["sampled"] = toks
        rec["finished"] = [r.id for r in dec if r.is_finished()]
        rec["free_blocks"] = [b.block_id for b in kvm.free_block_queue]
        out.append(rec)
    return out, outcome, {r.id: r.token_ids for r in reqs}


SCENARIOS = [sc["name"] for sc in _load()]


@pytest.mark.parametrize("name", SCENARIOS)
def test_host_trace_matches_reference(name):
    sc = next(s for s in _load() if s["name"] == name)
    steps, outcome, final = replay(sc)
    assert outcome == sc["outcome"]
    assert len(steps) == len(sc["steps"])
    for i, (got, ref) in enumerate(zip(steps, sc["steps"])):
        for key in ("decode_ids", "prefill_ids", "waiting_ids", "running_ids", "sampled",
                    "finished", "free_blocks"):
            assert got[key] == ref[key], f"step {i} {key}"
        for phase in ("decode", "prefill"):
            assert (phase in got) == (phase in ref), f"step {i} {phase}"
            if phase in ref:
                for k, v in ref[phase].items():
                    np.testing.assert_array_equal(np.asarray(got[phase][k]), np.asarray(v),
                                                  err_msg=f"step {i} {phase}.{k}")
    assert {int(k): v for k, v in sc["final_tokens"].items()} == final


def test_goldens_cover_quirks():
    """The goldens exercise the reference behaviours this build must keep."""
    data = {s["name"]: s for s in _load()}
    assert data["preempt_assert"]["outcome"].startswith("assert")
    assert data["preempt_stall"]["outcome"] == "step_cap"
    # a decode step right after a block-boundary allocation stores the token in
    # the LAST block (model_runner.py:282-284), not the block of its position
    c1 = data["c1"]
    seen = False
    for st in c1["steps"]:
        if "decode" not in st:
            continue
        d = st["decode"]
        for b, pos in enumerate(d["positions"][:len(st["decode_ids"])]):
            row = [x for x in d["block_tables"][b] if x >= 0]
            if (pos + 1) % 16 == 0 and len(row) * 16 > pos + 1:
                assert d["slot_mapping"][b] == row[-1] * 16 + pos % 16
                assert row[-1] != row[pos // 16]
                seen = True
    assert seen
