"""End-to-end engine on the GPU: C1 greedy decoding vs the oracle, the
reference-signature attention boundary, preemption and tensor-parallel setup."""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "host_traces.json")


def _c1():
    with open(GOLDEN) as f:
        return next(s for s in json.load(f) if s["name"] == "c1")


@pytest.fixture(scope="module", params=[0, 64], ids=["cublas", "fused_gemm"])
def c1_run(request):
    """Qwen3-0.6B, random weights (seed 0, drawn on the CPU), the C1 prompts;
    projections on cuBLAS + separate K3 / SiLU launches, or (fused_gemm) on
    this library's tcgen05 GEMMs with fused epilogues for forwards of <= 64 rows."""
    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import PRESETS, Qwen3Weights
    from vllm_b200.src.engine import Engine
    from vllm_b200.src.request import Request
    sc = _c1()
    cfg = PRESETS["Qwen3-0.6B"]
    dev = torch.device("cuda", 0)
    weights = Qwen3Weights(cfg, dev, seed=0, gen_device="cpu")
    Request.reset_ids()
    eng = Engine(Config(model="Qwen3-0.6B", fused_gemm_max_rows=request.param, **sc["config"]),
                 dev, model_config=cfg, weights=weights, max_slots=16)
    outs = eng.generate(sc["prompts"], SamplingParams(temperature=0.0, max_new_tokens=32,
                                                      ignore_eos=True))
    return sc, cfg, weights, eng, outs


def test_c1_engine_runs_and_schedules_like_reference(c1_run):
    sc, cfg, weights, eng, outs = c1_run
    assert [len(o) for o in outs] == [32] * 4
    assert eng.stats["steps"] == len(sc["steps"])           # same step count as the reference
    # block ids the engine used are the reference's (same FIFO pool)
    assert [b.block_id for b in eng.kv.free_block_queue] == sc["steps"][-1]["free_blocks"]


def _bf16_ulp(x: float) -> float:
    return 2.0 ** (math.floor(math.log2(max(abs(x), 2.0 ** -10))) - 7)


def test_c1_greedy_tokens_vs_oracle(c1_run):
    """Greedy tokens of the first 32 steps of all 4 C1 requests against the
    oracle's restatement of the reference forward (bf16 q scaling as the
    reference, compat=True).

    Every one of the 4 x 32 steps is checked: the oracle replays the ENGINE's
    tokens (teacher forcing) and at each step the engine's token must be the
    oracle's argmax, or -- logits are bf16, so accumulation order can move a
    logit by an ulp -- within 2 bf16 ulps of the oracle's top logit (a near
    tie). The free-running agreement (oracle feeding back its own argmax) is
    reported too."""
    from oracle.qwen3 import OracleQwen3, greedy_replay
    sc, cfg, weights, eng, outs = c1_run
    W = weights.full_numpy()
    nb, bs = sc["config"]["num_blocks"], sc["config"]["block_size"]
    _, steps = greedy_replay(OracleQwen3(cfg, W, nb, bs), sc, sc["prompts"], forced=outs)
    n_rows = sum(len(s) for s in steps)
    assert n_rows == 4 * 32
    seen = {r: 0 for r in range(4)}
    identical, ties = 0, []
    for st, step in zip((s for s in sc["steps"] if "decode" in s), steps):
        for r, (top, top_logit, gap, chosen) in zip(st["decode_ids"], step):
            k = seen[r]
            seen[r] += 1
            if outs[r][k] == top:
                identical += 1
                continue
            deficit = top_logit - chosen
            ties.append((r, k, deficit / _bf16_ulp(top_logit)))
            assert deficit <= 2 * _bf16_ulp(top_logit) + 1e-9, (
                f"request {r} step {k}: engine token {outs[r][k]} is {deficit:.5f} below the "
                f"oracle's top logit {top_logit:.4f} (top {top})")
    free, _ = greedy_replay(OracleQwen3(cfg, W, nb, bs), sc, sc["prompts"])
    prefix = []
    for r in range(4):
        ref = free[r][len(sc["prompts"][r]):]
        n = 0
        while n < 32 and outs[r][n] == ref[n]:
            n += 1
        prefix.append(n)
    print(f"greedy parity: {identical}/128 steps pick the oracle's argmax; near ties "
          f"(request, step, ulps below the top): {ties}; free-running identical prefix per "
          f"request: {prefix} (sum {sum(prefix)}/128)")


def test_attention_boundary_reference_signature():
    """attention(kv_cache, q, k, v, metadata) of vllm/model/qwen3.py:172-218."""
    from vllm_b200.model.qwen3 import (DecodeAttentionMetadata, PrefillAttentionMetadata,
                                       attention)
    rng = np.random.default_rng(4)
    nb, bs, Hkv, Hq, D = 32, 16, 8, 32, 128
    t = lambda x, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(x)).to(dt).cuda()
    cache = np.zeros((2, nb, bs, Hkv, D), np.float32)
    # prefill of two sequences (20 and 37 tokens), padded to 64
    lens = [20, 37]
    blocks = [[3, 9], [0, 7, 12]]
    slots, pos = [], []
    for L, blk in zip(lens, blocks):
        slots += [blk[i // bs] * bs + i % bs for i in range(L)]
        pos += list(range(L))
    T = 64
    slots += [-1] * (T - len(slots))
    pos += [0] * (T - len(pos))
    q = bf16(rng.standard_normal((T, Hq, D)))
    k = bf16(rng.standard_normal((T, Hkv, D)))
    v = bf16(rng.standard_normal((T, Hkv, D)))
    # bucket padding rows are identical (token 0 at position 0) and all write slot -1
    k[57:], v[57:] = k[57], v[57]
    bt = np.full((4, 8), -1, np.int32)
    for i, blk in enumerate(blocks):
        bt[i, :len(blk)] = blk
    cu = np.array([0, 20, 57, 57, 57], np.int32)
    kc, vc = cache[0].copy(), cache[1].copy()
    from oracle import kv_store as okv
    okv.update_kv_cache(kc, vc, np.asarray(slots), k, v)
    ref = oatt.prefill_attention(q, kc, vc, bt, cu[:3], np.array(lens), 1 / math.sqrt(D))
    d_cache = t(cache)
    meta = PrefillAttentionMetadata(t(pos, torch.int32), t(slots, torch.int32),
                                    t(bt, torch.int32), t(cu, torch.int32), t(cu, torch.int32),
                                    37, 37, 64, num_seqs=2)
    d_cache, out = attention(d_cache, t(q), t(k), t(v), meta)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
    np.testing.assert_array_equal(d_cache.float().cpu().numpy()[0], kc)
    # decode of the same two sequences, one new token each
    qd = bf16(rng.standard_normal((2, Hq, D)))
    kd = bf16(rng.standard_normal((2, Hkv, D)))
    vd = bf16(rng.standard_normal((2, Hkv, D)))
    dslots = np.array([blocks[0][20 // bs] * bs + 20 % bs, blocks[1][37 // bs] * bs + 37 % bs],
                      np.int32)
    okv.update_kv_cache(kc, vc, dslots, kd, vd)
    ctx = np.array([21, 38], np.int32)
    ref = oatt.decode_attention(qd, kc, vc, bt[:2], ctx, 1 / math.sqrt(D))
    dmeta = DecodeAttentionMetadata(t([20, 37], torch.int32), t(dslots, torch.int32),
                                    t(bt[:2], torch.int32), t(ctx, torch.int32))
    d_cache, out = attention(d_cache, t(qd), t(kd), t(vd), dmeta)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3


def test_engine_preemption_completes_without_compat():
    """A pool too small for all requests forces tail preemption and re-prefill;
    with compat=False (finished requests free their blocks) the run completes."""
    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
    from vllm_b200.src.engine import Engine
    cfg = Qwen3Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=16, vocab_size=1000, tie_word_embeddings=True)
    dev = torch.device("cuda", 0)
    w = Qwen3Weights(cfg, dev, seed=1)
    eng = Engine(Config(model="tiny", max_num_batched_tokens=256, max_num_seqs=3,
                        num_blocks=11, block_size=16, compat=False), dev, model_config=cfg,
                 weights=w, max_slots=16)
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 1000, n).tolist() for n in (46, 17, 20, 28, 19, 58)]
    outs = eng.generate(prompts, SamplingParams(temperature=0, max_new_tokens=27,
                                                ignore_eos=True))
    assert [len(o) for o in outs] == [27] * 6
    assert eng.stats["prefill_tokens"] > sum(len(p) for p in prompts)   # re-prefills happened


def test_engine_loads_a_local_hf_checkpoint(tmp_path):
    """Config(model=<directory>) reads config.json and the safetensors weights."""
    import json as _json

    from safetensors.torch import save_file

    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
    from vllm_b200.src.engine import Engine
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      tie_word_embeddings=False)
    w = Qwen3Weights(cfg, torch.device("cpu"), seed=4)
    D, Hq, Hkv, I = cfg.head_dim, 4, 2, cfg.intermediate_size
    t = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.norm,
         "lm_head.weight": w.lm_head}
    for l, lw in enumerate(w.layers):
        p = f"model.layers.{l}."
        q, k, v = torch.split(lw.w_qkv, [Hq * D, Hkv * D, Hkv * D])
        g, u = torch.split(lw.w_gate_up, [I, I])
        t.update({p + "self_attn.q_proj.weight": q, p + "self_attn.k_proj.weight": k,
                  p + "self_attn.v_proj.weight": v, p + "self_attn.o_proj.weight": lw.w_o,
                  p + "self_attn.q_norm.weight": lw.q_norm,
                  p + "self_attn.k_norm.weight": lw.k_norm,
                  p + "mlp.gate_proj.weight": g, p + "mlp.up_proj.weight": u,
                  p + "mlp.down_proj.weight": lw.w_down, p + "input_layernorm.weight": lw.ln1,
                  p + "post_attention_layernorm.weight": lw.ln2})
    save_file({k: x.clone().contiguous() for k, x in t.items()},
              str(tmp_path / "model.safetensors"))
    with open(tmp_path / "config.json", "w") as f:
        _json.dump(dict(vocab_size=512, hidden_size=256, intermediate_size=512,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                        tie_word_embeddings=False), f)
    dev = torch.device("cuda", 0)
    conf = dict(max_num_batched_tokens=128, max_num_seqs=2, num_blocks=32, block_size=16,
                compat=False)
    sp = SamplingParams(temperature=0, max_new_tokens=6, ignore_eos=True)
    prompts = [[1, 2, 3, 4, 5], list(range(40, 77))]
    a = Engine(Config(model=str(tmp_path), **conf), dev, max_slots=4).generate(prompts, sp)
    b = Engine(Config(model="x", **conf), dev, model_config=cfg,
               weights=Qwen3Weights(cfg, dev, seed=4, gen_device="cpu"),
               max_slots=4).generate(prompts, sp)
    assert a == b


def test_lookahead_scheduling_matches_synchronous_steps():
    """generate() with async_scheduling (step k+1 enqueued before step k's
    tokens are read) gives the same tokens as the synchronous loop."""
    from vllm_b200 import Config, SamplingParams
    from vllm_b200.model.qwen3 import Qwen3Config, Qwen3Weights
    from vllm_b200.src.engine import Engine
    cfg = Qwen3Config(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=16, vocab_size=1000, tie_word_embeddings=True)
    dev = torch.device("cuda", 0)
    w = Qwen3Weights(cfg, dev, seed=6)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 1000, n).tolist() for n in (46, 17, 20, 28, 19, 58, 5)]
    outs = []
    for async_on in (False, True):
        eng = Engine(Config(model="tiny", max_num_batched_tokens=256, max_num_seqs=4,
                            num_blocks=40, block_size=16, compat=False,
                            async_scheduling=async_on), dev, model_config=cfg, weights=w,
                     max_slots=16)
        assert eng.async_scheduling == async_on
        outs.append(eng.generate(prompts, SamplingParams(temperature=0, max_new_tokens=21,
                                                         ignore_eos=True)))
    assert outs[0] == outs[1]
