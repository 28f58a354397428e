"""K4 GPU metadata builder vs the reference's own packing (golden traces).

Every step of every golden scenario is replayed through this build's host
scheduler; the scheduled requests' token ids and block lists live only in the
device tables (uploaded as deltas), and vj_build_metadata must reproduce the
reference's prepare_prefill / prepare_decode arrays bit for bit."""
import numpy as np
import pytest
import torch

from test_host_golden import _load, replay

pytestmark = pytest.mark.gpu


def _np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("name", [sc["name"] for sc in _load()])
def test_gpu_metadata_matches_reference_packing(name):
    from vllm_b200.kernels.metadata import DeviceTables
    sc = next(s for s in _load() if s["name"] == name)
    dev = torch.device("cuda", 0)
    cfg = sc["config"]
    max_len = 4096
    width = (cfg["max_num_batched_tokens"] + cfg["block_size"] - 1) // cfg["block_size"]
    tables = DeviceTables(64, max_len, width + 4, cfg["block_size"], dev)
    slot_of = {}
    known_tokens = {}
    checked = {"decode": 0, "prefill": 0}

    def on_step(rec, dec, pre, kvm, c):
        i = len(getattr(on_step, "seen", []))
        on_step.seen = getattr(on_step, "seen", []) + [1]
        ref = sc["steps"][i]
        # upload deltas: new requests' tokens, changed block lists
        tok_rows, blk_rows = [], []
        for r in dec + pre:
            if r.id not in slot_of:
                slot_of[r.id] = len(slot_of)
            s = slot_of[r.id]
            have = known_tokens.get(r.id, 0)
            if have < len(r.token_ids):
                tok_rows.append((s, have, r.token_ids[have:]))
                known_tokens[r.id] = len(r.token_ids)
        for rid in sorted(kvm.dirty):
            if rid in slot_of:
                blk_rows.append((slot_of[rid], kvm.req_to_blocks.get(rid, [])))
        kvm.dirty.clear()
        tables.set_tokens(tok_rows)
        tables.set_blocks([(s, [b.block_id for b in blks]) for s, blks in blk_rows])
        if dec:
            m = tables.build_decode([slot_of[r.id] for r in dec], [len(r) for r in dec], width)
            g = ref["decode"]
            for k in ("input_ids", "positions", "slot_mapping", "block_tables", "context_lens"):
                np.testing.assert_array_equal(_np(getattr(m, k)), np.asarray(g[k]),
                                              err_msg=f"{name} step {i} decode.{k}")
            checked["decode"] += 1
        if pre:
            m = tables.build_prefill([slot_of[r.id] for r in pre], [len(r) for r in pre],
                                     c.max_num_seqs, width)
            g = ref["prefill"]
            for k, gk in (("input_ids", "input_ids"), ("positions", "positions"),
                          ("slot_mapping", "slot_mapping"), ("block_tables", "block_tables"),
                          ("cu_seqlens_q", "cu_seqlens_q")):
                np.testing.assert_array_equal(_np(getattr(m, k)), np.asarray(g[gk]),
                                              err_msg=f"{name} step {i} prefill.{k}")
            assert m.max_seqlen_bucket == g["max_seqlen_bucket"]
            assert m.max_seqlen_q == g["max_seqlen_q"]
            checked["prefill"] += 1
        tables.check()

    replay(sc, on_step)
    assert checked["decode"] + checked["prefill"] > 0


def test_argmax_append_first_index_on_ties():
    from vllm_b200.kernels.metadata import DeviceTables
    dev = torch.device("cuda", 0)
    t = DeviceTables(8, 64, 4, 16, dev)
    V = 151936
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    logits = torch.randn((5, V), generator=g, device=dev).to(torch.bfloat16)
    logits[1, 100] = 50.0
    logits[1, 7] = 50.0                    # tie: first index wins
    logits[2, :] = -1.0                    # all equal -> 0
    logits[3, V - 1] = 99.0
    slots = torch.tensor([0, 1, 2, 3, 4], dtype=torch.int32, device=dev)
    lens = torch.tensor([3, 5, 0, 63, 10], dtype=torch.int32, device=dev)
    out = t.argmax_append(logits, slots, lens)
    ref = torch.argmax(logits.float(), dim=-1)
    got = out.cpu().numpy()
    assert got[1] == 7 and got[2] == 0 and got[3] == V - 1
    np.testing.assert_array_equal(got[[0, 4]], ref.cpu().numpy()[[0, 4]])
    tok = t.tokens.cpu().numpy()
    for r, (s, L) in enumerate(zip(slots.tolist(), lens.tolist())):
        assert tok[s, L] == got[r]
