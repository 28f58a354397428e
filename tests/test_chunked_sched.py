"""Chunked prefill on the host (CPU): the token-budget scheduler and the
oracle's ranges packing.

* prepare_ranges with every sequence starting at position 0 is the
  reference's prepare_prefill packing: checked on every prefill step of the
  golden traces (recorded from the reference's own code).
* ChunkedScheduler invariants on random workloads, with a pool small enough
  to force preemption: token budget and sequence cap per step, each row
  continues exactly where its request's cache ends, blocks cover every
  computed position and are never shared, every request completes with its
  max_new_tokens, and finished requests give all blocks back.
"""
import numpy as np
import pytest

from oracle import host as ohost
from test_host_golden import _load, replay


@pytest.mark.parametrize("name", [sc["name"] for sc in _load()])
def test_ranges_from_zero_is_reference_prefill_packing(name):
    sc = next(s for s in _load() if s["name"] == name)
    checked = []

    def on_step(rec, dec, pre, kvm, cfg):
        i = len(checked)
        checked.append(0)
        ref = sc["steps"][i].get("prefill")
        if not pre or ref is None:
            return
        got = ohost.prepare_ranges([r.token_ids for r in pre], [kvm.block_ids(r) for r in pre],
                                   [0] * len(pre), [len(r) for r in pre], cfg.block_size,
                                   cfg.max_num_seqs, cfg.max_blocks_per_seq)
        for k in ("input_ids", "positions", "slot_mapping", "block_tables", "cu_seqlens_q"):
            np.testing.assert_array_equal(got[k], np.asarray(ref[k]), err_msg=f"step {i} {k}")
        ctx = got["context_lens"]
        np.testing.assert_array_equal(ctx[:len(pre)], [len(r) for r in pre])
        assert not ctx[len(pre):].any()
        checked[-1] = 1

    replay(sc, on_step)
    if name != "preempt_assert":
        assert sum(checked) > 0


def _drive(prompt_lens, max_new, budget, max_seqs, num_blocks, bs, seed=0, eos=None):
    from vllm_b200.config import Config
    from vllm_b200.sampling_params import SamplingParams
    from vllm_b200.src.kv_cache_manager import KVCacheManager
    from vllm_b200.src.request import Request
    from vllm_b200.src.scheduler import ChunkedScheduler

    Request.reset_ids()
    cfg = Config(model="synthetic", max_num_batched_tokens=budget, max_num_seqs=max_seqs,
                 num_blocks=num_blocks, block_size=bs, compat=False,
                 enable_chunked_prefill=True)
    kv = KVCacheManager(num_blocks, bs)
    sched = ChunkedScheduler(cfg, kv)
    rng = np.random.default_rng(seed)
    reqs = [Request(rng.integers(0, 1000, n).tolist(),
                    SamplingParams(temperature=0, max_new_tokens=max_new, ignore_eos=eos is None),
                    eos if eos is not None else -1) for n in prompt_lens]
    for r in reqs:
        sched.add(r)
    trace, preempted = [], []
    plain = sched._preempt

    def counting(req):
        preempted.append(req.id)
        plain(req)

    sched._preempt = counting
    while not sched.is_finished():
        assert len(trace) < 10000, "no progress"
        batch = sched.schedule()
        assert batch, "empty step while requests remain"
        assert sum(n for _, n in batch) <= budget
        assert len(batch) <= max_seqs
        assert len({r.id for r, _ in batch}) == len(batch)
        owned = []
        for r, n in batch:
            assert n >= 1
            assert r.num_computed_tokens + n <= len(r)
            blocks = kv.block_ids(r)
            assert len(blocks) * bs >= r.num_computed_tokens + n
            owned += blocks
        assert len(owned) == len(set(owned)), "a block owned twice"
        sampled = {}
        for r, n in batch:
            if r.num_computed_tokens + n == len(r):
                t = int(rng.integers(0, 1000)) if eos is None else eos
                r.token_ids.append(t)
                r.num_completion_tokens += 1
                sampled[r.id] = t
        sched.postprocess(batch, sampled)
        trace.append(([(r.id, r.num_computed_tokens, n) for r, n in batch],
                      [b.block_id for b in kv.free_block_queue]))
    for r in reqs:
        want = 1 if eos is not None else max_new
        assert r.num_completion_tokens == want
        assert r.num_computed_tokens == len(r) - 1
    assert len(kv.free_block_queue) == num_blocks
    return trace, len(preempted)


def test_chunked_scheduler_invariants_and_completion():
    lens = [300, 17, 64, 129, 5, 250, 33, 90]
    trace, pre = _drive(lens, max_new=20, budget=96, max_seqs=4, num_blocks=64, bs=16)
    # prompts longer than the budget were split over several steps
    chunks = [n for step, _ in trace for _, _, n in step if n > 1]
    assert max(chunks) <= 96 and len(chunks) > len(lens)
    # some step mixed decode rows with prompt chunks
    assert any(any(n == 1 for _, _, n in s) and any(n > 1 for _, _, n in s) for s, _ in trace)


def test_chunked_scheduler_preempts_on_a_small_pool():
    lens = [120, 100, 90, 80, 110, 70]
    trace, pre = _drive(lens, max_new=40, budget=64, max_seqs=6, num_blocks=24, bs=16, seed=3)
    assert pre > 0


def test_chunked_scheduler_eos_and_determinism():
    _drive([40, 50, 60], max_new=10, budget=32, max_seqs=2, num_blocks=16, bs=16, eos=7)
    a = _drive([200, 31, 77, 5], max_new=9, budget=48, max_seqs=3, num_blocks=20, bs=16, seed=5)
    b = _drive([200, 31, 77, 5], max_new=9, budget=48, max_seqs=3, num_blocks=20, bs=16, seed=5)
    assert a == b
