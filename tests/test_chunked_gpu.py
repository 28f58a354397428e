"""Chunked prefill mixed with decode on the GPU.

* K4 in ranges mode (vj_build_metadata, VJ_META_RANGES) against the
  oracle's prepare_ranges, bit for bit, plus the sampled-row tables.
* The engine with enable_chunked_prefill on a small Qwen3: prompts longer
  than the token budget are split into chunks that share forwards with decode
  rows; greedy tokens are checked against the oracle replaying the same
  recorded schedule (same near-tie rule as the C1 test).
"""
import math

import numpy as np
import pytest
import torch

from oracle import host as ohost

pytestmark = pytest.mark.gpu


def test_ranges_metadata_matches_oracle():
    from vllm_b200.kernels.metadata import DeviceTables
    dev = torch.device("cuda", 0)
    bs, width, max_len = 16, 24, 384
    tables = DeviceTables(32, max_len, width, bs, dev)
    rng = np.random.default_rng(11)
    pool = rng.permutation(200).tolist()
    lens = [300, 17, 64, 129, 5, 250]
    toks, blocks = [], []
    for i, L in enumerate(lens):
        toks.append(rng.integers(0, 50000, L).tolist())
        nb = (L + bs - 1) // bs
        blocks.append([pool.pop() for _ in range(nb)])
    tables.set_tokens([(3 * i, 0, t) for i, t in enumerate(toks)])
    tables.set_blocks([(3 * i, b) for i, b in enumerate(blocks)])
    starts = [0, 16, 63, 100, 0, 249]
    ns = [37, 1, 1, 29, 5, 1]
    sample = [1, 2, 4, 5]
    m = tables.build_ranges([3 * i for i in range(len(lens))], starts, ns, width, sample,
                            bucket_batch=8)
    tables.check()
    ref = ohost.prepare_ranges(toks, blocks, starts, ns, bs, 8, width)
    for k in ("input_ids", "positions", "slot_mapping", "block_tables", "cu_seqlens_q",
              "context_lens"):
        np.testing.assert_array_equal(getattr(m, k).cpu().numpy(), ref[k], err_msg=k)
    cu = ref["cu_seqlens_q"]
    np.testing.assert_array_equal(m.sample_rows.cpu().numpy(), [cu[s + 1] - 1 for s in sample])
    np.testing.assert_array_equal(m.sample_slots.cpu().numpy(), [3 * s for s in sample])
    np.testing.assert_array_equal(m.sample_lens.cpu().numpy(),
                                  [starts[s] + ns[s] for s in sample])
    assert m.max_new == 37 and m.num_tokens == sum(ns)


def test_chunked_engine_greedy_vs_oracle():
    from oracle.qwen3 import OracleQwen3, greedy_replay_chunked
    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
    from vllm_b200.src.engine import Engine
    from vllm_b200.src.request import Request
    cfg = Qwen3Config(vocab_size=4096, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=4)
    dev = torch.device("cuda", 0)
    w = Qwen3Weights(cfg, dev, seed=7, gen_device="cpu")
    nb, bs = 96, 16
    Request.reset_ids()
    eng = Engine(Config(model="tiny", max_num_batched_tokens=48, max_num_seqs=4,
                        num_blocks=nb, block_size=bs, max_model_len=256,
                        enable_chunked_prefill=True), dev, model_config=cfg, weights=w,
                 max_slots=16)
    eng.trace = []
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (100, 37, 70, 9, 130)]
    new = 12
    outs = eng.generate(prompts, SamplingParams(temperature=0, max_new_tokens=new,
                                                ignore_eos=True))
    assert [len(o) for o in outs] == [new] * len(prompts)
    assert len(eng.kv.free_block_queue) == nb
    steps = [st["batch"] for st in eng.trace]
    assert any(n > 1 and a > 0 for s in steps for _, a, n in s)          # chunk after a prefix
    assert any(any(n == 1 for *_, n in s) and any(n > 1 for *_, n in s) for s in steps)
    model = OracleQwen3(cfg, w.full_numpy(), nb, bs)
    tokens, gaps = greedy_replay_chunked(model, eng.trace, prompts)
    n_match, first = 0, None
    for r, p in enumerate(prompts):
        ref = tokens[r][len(p):]
        for i, (a, b) in enumerate(zip(outs[r], ref)):
            if a != b:
                first = (r, i) if first is None or i < first[1] else first
                break
            n_match += 1
    print(f"chunked greedy agreement {n_match}/{new * len(prompts)}; first divergence {first}")
    if first is not None:
        r, i = first
        # the step at which request r sampled its i-th token
        k = -1
        for s, g in enumerate(gaps):
            if r in g:
                k += 1
                if k == i:
                    _, top, gap = g[r]
                    break
        ulp = 2.0 ** (math.floor(math.log2(max(abs(top), 2.0 ** -10))) - 7)
        assert gap <= 4 * ulp + 1e-9, f"request {r} diverged at token {i}, oracle gap {gap}"
    assert n_match >= new * len(prompts) // 2


def test_prefix_cached_engine_greedy_vs_oracle():
    """Prompts sharing stems reuse cached KV blocks (written by earlier
    requests, possibly after those finished); the oracle replays the recorded
    schedule with the same block tables, so shared blocks hold the KV it
    computed for the first request."""
    from oracle.qwen3 import OracleQwen3, greedy_replay_chunked
    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
    from vllm_b200.src.engine import Engine
    from vllm_b200.src.request import Request
    cfg = Qwen3Config(vocab_size=4096, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=4)
    dev = torch.device("cuda", 0)
    w = Qwen3Weights(cfg, dev, seed=9, gen_device="cpu")
    nb, bs = 64, 16
    Request.reset_ids()
    eng = Engine(Config(model="tiny", max_num_batched_tokens=64, max_num_seqs=3,
                        num_blocks=nb, block_size=bs, max_model_len=256,
                        enable_chunked_prefill=True, enable_prefix_caching=True), dev,
                 model_config=cfg, weights=w, max_slots=16)
    eng.trace = []
    rng = np.random.default_rng(3)
    stem = rng.integers(0, cfg.vocab_size, 90).tolist()
    prompts = [stem + rng.integers(0, cfg.vocab_size, n).tolist() for n in (5, 30, 1, 12, 40)]
    prompts.append(stem[:64])                             # whole-block prefix of the stem
    new = 8
    outs = eng.generate(prompts, SamplingParams(temperature=0, max_new_tokens=new,
                                                ignore_eos=True))
    assert eng.scheduler.prefix_hit_tokens >= 4 * 80
    assert [len(o) for o in outs] == [new] * len(prompts)
    model = OracleQwen3(cfg, w.full_numpy(), nb, bs)
    tokens, gaps = greedy_replay_chunked(model, eng.trace, prompts)
    n_match, first = 0, None
    for r, p in enumerate(prompts):
        for i, (a, b) in enumerate(zip(outs[r], tokens[r][len(p):])):
            if a != b:
                first = (r, i) if first is None or i < first[1] else first
                break
            n_match += 1
    print(f"prefix-cached greedy agreement {n_match}/{new * len(prompts)}; first {first}")
    if first is not None:
        r, i = first
        k = -1
        for g in gaps:
            if r in g:
                k += 1
                if k == i:
                    _, top, gap = g[r]
                    break
        ulp = 2.0 ** (math.floor(math.log2(max(abs(top), 2.0 ** -10))) - 7)
        assert gap <= 4 * ulp + 1e-9, f"request {r} diverged at token {i}, oracle gap {gap}"
    assert n_match >= new * len(prompts) // 2
