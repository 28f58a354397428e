"""The engine's one-step-lookahead loop (async_scheduling) on the CPU with a
fake model runner whose token at (request, position) is a fixed function, so
any schedule must produce the same completions: the lookahead loop must match
the synchronous step() loop exactly, including requests that stop at EOS one
step before the lookahead learns it, and preemptions on a small pool."""
import numpy as np
import pytest

EOS = 0


def _tok(rid, pos):
    if (rid * 3 + pos) % 17 == 0:
        return EOS
    return 1 + (rid * 31 + pos * 7) % 50


class FakePending:
    def __init__(self, toks):
        self.toks = toks

    def collect(self):
        return list(self.toks)


class FakeRunner:
    """Stands in for ModelRunner: tokens from _tok, no device."""

    def __init__(self):
        self.launches = 0

    def release(self, r):
        r.slot = -1

    def _tokens(self, decode):
        return [_tok(r.id, len(r)) for r in decode]

    def launch(self, decode, prefill, live, stats):
        self.launches += 1
        return FakePending(self._tokens(decode)) if decode else None

    def run(self, decode, prefill, live, stats):
        out = self._tokens(decode)
        for r, t in zip(decode, out):
            r.token_ids.append(t)
            r.num_completion_tokens += 1
        return out


def _engine(async_on, num_blocks):
    from vllm_b200.config import Config
    from vllm_b200.src.engine import Engine
    from vllm_b200.src.kv_cache_manager import KVCacheManager
    from vllm_b200.src.scheduler import Scheduler
    cfg = Config(model="fake", max_num_batched_tokens=256, max_num_seqs=4,
                 num_blocks=num_blocks, block_size=16, compat=False,
                 async_scheduling=async_on)
    e = object.__new__(Engine)
    e.config, e.tokenizer, e.eos_token_id, e.tp_comm, e.trace = cfg, None, EOS, None, None
    e.kv = KVCacheManager(num_blocks, 16)
    e.scheduler = Scheduler(cfg, e.kv)
    e.runner = FakeRunner()
    e.live = {}
    e.stats = {k: 0 for k in ("steps", "decode_tokens", "prefill_tokens", "decode_steps",
                              "decode_ctx_tokens", "h2d_bytes", "d2h_bytes")}
    e.stats.update(decode_s=0.0, prefill_s=0.0)
    return e


@pytest.mark.parametrize("num_blocks", [64, 13, 16])
def test_lookahead_loop_matches_synchronous_loop(num_blocks):
    from vllm_b200.sampling_params import SamplingParams
    from vllm_b200.src.request import Request
    rng = np.random.default_rng(1)
    prompts = [rng.integers(1, 100, int(n)).tolist() for n in rng.integers(5, 60, 9)]
    params = [SamplingParams(temperature=0, max_new_tokens=int(m), ignore_eos=bool(i % 3 == 0))
              for i, m in enumerate(rng.integers(3, 40, 9))]
    outs, preempted = [], []
    for async_on in (False, True):
        Request.reset_ids()
        e = _engine(async_on, num_blocks)
        assert e.async_scheduling == async_on
        count = []
        plain = e.scheduler.preempt
        e.scheduler.preempt = lambda r, plain=plain, count=count: (count.append(r.id), plain(r))
        preempted.append(len(count))
        outs.append(e.generate(prompts, params))
        assert e.scheduler.is_finished() and not e.live
        assert len(e.kv.free_block_queue) == num_blocks
        assert all(-1 not in o for o in outs[-1])
        preempted[-1] = len(count)
    assert outs[0] == outs[1]
    if num_blocks < 64:
        assert min(preempted) > 0                  # the small pool did preempt
    # EOS stops and max-token stops both occurred
    assert any(o and o[-1] == EOS for o in outs[0])
    assert any(len(o) == p.max_new_tokens for o, p in zip(outs[0], params))
