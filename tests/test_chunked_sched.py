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


def _prefix_setup(num_blocks=40, budget=512):
    from vllm_b200.config import Config
    from vllm_b200.src.kv_cache_manager import KVCacheManager
    from vllm_b200.src.request import Request
    from vllm_b200.src.scheduler import ChunkedScheduler
    Request.reset_ids()
    cfg = Config(model="synthetic", max_num_batched_tokens=budget, max_num_seqs=8,
                 num_blocks=num_blocks, block_size=16, compat=False,
                 enable_chunked_prefill=True, enable_prefix_caching=True)
    kv = KVCacheManager(num_blocks, 16)
    return kv, ChunkedScheduler(cfg, kv)


def _req(tokens, new=4):
    from vllm_b200.sampling_params import SamplingParams
    from vllm_b200.src.request import Request
    return Request(tokens, SamplingParams(temperature=0, max_new_tokens=new, ignore_eos=True), -1)


def _step(sched, tok=1):
    batch = sched.schedule()
    sampled = {}
    for r, n in batch:
        if r.num_computed_tokens + n == len(r):
            r.token_ids.append(tok)
            r.num_completion_tokens += 1
            sampled[r.id] = tok
    sched.postprocess(batch, sampled)
    return batch


def test_prefix_cache_shares_full_blocks_and_survives_finish():
    kv, sched = _prefix_setup()
    shared = list(range(1000, 1100))                       # 100 tokens: 6 full blocks
    r1 = _req(shared + [1, 2, 3])
    sched.add(r1)
    _step(sched)                                           # r1 prefilled (103 tokens)
    r2 = _req(shared + [7, 8])
    sched.add(r2)
    batch = _step(sched)
    (_, n1), (b2, n2) = batch
    assert b2 is r2 and n2 == 102 - 96                     # starts after 6 cached blocks
    assert kv.block_ids(r2)[:6] == kv.block_ids(r1)[:6]
    assert all(b.ref_count == 2 for b in kv.get_block_table(r1)[:6])
    assert sched.prefix_hit_tokens == 96
    while not sched.is_finished():
        _step(sched)
    assert len(kv.free_block_queue) == kv.num_blocks       # all released ...
    assert len(kv.cached) >= 6                             # ... but still cached
    r3 = _req(shared)                                      # exact prefix, 100 tokens
    sched.add(r3)
    batch = _step(sched)
    assert batch[0][1] == 100 - 96 and sched.prefix_hit_tokens == 192


def test_prefix_cache_never_skips_the_last_token_and_evicts_on_reuse():
    kv, sched = _prefix_setup(num_blocks=12)
    p = list(range(64))                                    # exactly 4 full blocks
    r1 = _req(p, new=1)
    sched.add(r1)
    while not sched.is_finished():
        _step(sched)
    r2 = _req(p, new=1)
    sched.add(r2)
    batch = _step(sched)
    assert batch[0][1] == 16                               # 3 blocks hit, last block recomputed
    while not sched.is_finished():
        _step(sched)
    # a large unrelated prompt takes every free block: the cached ones are evicted
    r3 = _req(list(range(5000, 5000 + 11 * 16 - 1)), new=1)
    sched.add(r3)
    _step(sched)
    assert all(b.hash is None or kv.cached.get(b.hash) is b for b in kv.blocks)
    hits = kv.lookup_prefix(_req(p), 10)
    assert len(hits) < 3


def test_prefix_cache_invariants_under_pressure():
    """Random prompts drawn from a few shared stems on a small pool: budget and
    seat caps hold, shared blocks are only full cached blocks, every request
    completes and all blocks return to the free queue."""
    kv, sched = _prefix_setup(num_blocks=48, budget=96)
    rng = np.random.default_rng(4)
    stems = [rng.integers(0, 1000, 70).tolist() for _ in range(3)]
    reqs = []
    for i in range(14):
        tail = rng.integers(0, 1000, int(rng.integers(1, 40))).tolist()
        r = _req(stems[i % 3][:int(rng.integers(10, 71))] + tail, new=int(rng.integers(1, 12)))
        reqs.append(r)
        sched.add(r)
    steps = 0
    while not sched.is_finished():
        steps += 1
        assert steps < 5000
        batch = _step(sched)
        assert sum(n for _, n in batch) <= 96
        owners = {}
        for r in sched.running:
            for b in kv.get_block_table(r):
                owners.setdefault(b.block_id, []).append(r)
        for bid, rs in owners.items():
            if len(rs) > 1:
                b = kv.blocks[bid]
                assert b.hash is not None and b.ref_count == len(rs)
    assert all(r.num_completion_tokens == r.max_new_tokens for r in reqs)
    assert len(kv.free_block_queue) == kv.num_blocks
    assert sched.prefix_hit_tokens > 0


def test_prefix_cache_hash_collision_is_not_a_hit():
    """A cached block is reused only if its tokens and its parent key match,
    not on the hash alone: force every chained hash to collide and check that
    a different prompt gets no hit while the same prompt still does."""
    kv, sched = _prefix_setup()
    kv.block_hashes = lambda token_ids, n, known=None: [7 + i for i in range(n)]
    p = list(range(200, 264))                              # 4 full blocks
    r1 = _req(p, new=1)
    sched.add(r1)
    while not sched.is_finished():
        _step(sched)
    assert len(kv.lookup_prefix(_req(p), 10)) == 4        # same tokens: hit
    other = list(range(900, 964))                          # same (forced) keys, other tokens
    assert kv.lookup_prefix(_req(other), 10) == []
    mixed = p[:32] + other[32:]                            # first two blocks match only
    assert len(kv.lookup_prefix(_req(mixed), 10)) == 2
