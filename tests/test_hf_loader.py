"""Hugging Face checkpoint loading (CPU): a tiny Qwen3 saved with HF tensor
names, as one safetensors file and as an indexed 2-shard checkpoint, loads
into Qwen3Weights; at tensor-parallel degree 2 each rank holds exactly the
rows/columns of its KV heads and intermediate slice
(vllm/utils/hf_convert.py:30-198 maps the same names)."""
import json

import pytest
import torch

CFG = dict(vocab_size=96, hidden_size=64, intermediate_size=48, num_hidden_layers=2,
           num_attention_heads=4, num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6,
           rope_parameters={"rope_theta": 10000.0}, tie_word_embeddings=False)


def _tensors():
    g = torch.Generator().manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g).bfloat16()
    H, D, I = CFG["hidden_size"], CFG["head_dim"], CFG["intermediate_size"]
    Hq, Hkv = CFG["num_attention_heads"], CFG["num_key_value_heads"]
    t = {"model.embed_tokens.weight": r(CFG["vocab_size"], H), "model.norm.weight": r(H),
         "lm_head.weight": r(CFG["vocab_size"], H)}
    for l in range(CFG["num_hidden_layers"]):
        p = f"model.layers.{l}."
        t.update({p + "self_attn.q_proj.weight": r(Hq * D, H),
                  p + "self_attn.k_proj.weight": r(Hkv * D, H),
                  p + "self_attn.v_proj.weight": r(Hkv * D, H),
                  p + "self_attn.o_proj.weight": r(H, Hq * D),
                  p + "self_attn.q_norm.weight": r(D), p + "self_attn.k_norm.weight": r(D),
                  p + "mlp.gate_proj.weight": r(I, H), p + "mlp.up_proj.weight": r(I, H),
                  p + "mlp.down_proj.weight": r(H, I),
                  p + "input_layernorm.weight": r(H), p + "post_attention_layernorm.weight": r(H)})
    return t


@pytest.mark.parametrize("sharded", [False, True])
def test_load_hf_checkpoint_with_tp_slices(tmp_path, sharded):
    from safetensors.torch import save_file

    from vllm_b200.model.hf_loader import config_from_hf, load_hf_weights
    t = _tensors()
    with open(tmp_path / "config.json", "w") as f:
        json.dump(CFG, f)
    if sharded:
        names = sorted(t)
        half = len(names) // 2
        parts = {"model-00001-of-00002.safetensors": names[:half],
                 "model-00002-of-00002.safetensors": names[half:]}
        wm = {}
        for fn, ks in parts.items():
            save_file({k: t[k].contiguous() for k in ks}, str(tmp_path / fn))
            wm.update({k: fn for k in ks})
        with open(tmp_path / "model.safetensors.index.json", "w") as f:
            json.dump({"weight_map": wm}, f)
    else:
        save_file(t, str(tmp_path / "model.safetensors"))
    cfg = config_from_hf(str(tmp_path))
    assert cfg.rope_theta == 10000.0 and cfg.head_dim == 32 and not cfg.tie_word_embeddings
    D = cfg.head_dim
    cpu = torch.device("cpu")
    for tp in (1, 2):
        for rank in range(tp):
            w = load_hf_weights(str(tmp_path), cpu, rank, tp)
            hq, hkv, il = 4 // tp, 2 // tp, 48 // tp
            qs = slice(rank * hq * D, (rank + 1) * hq * D)
            ks = slice(rank * hkv * D, (rank + 1) * hkv * D)
            isl = slice(rank * il, (rank + 1) * il)
            for l, lw in enumerate(w.layers):
                p = f"model.layers.{l}."
                assert torch.equal(lw.w_qkv, torch.cat([t[p + "self_attn.q_proj.weight"][qs],
                                                        t[p + "self_attn.k_proj.weight"][ks],
                                                        t[p + "self_attn.v_proj.weight"][ks]]))
                assert torch.equal(lw.w_o, t[p + "self_attn.o_proj.weight"][:, qs])
                assert torch.equal(lw.w_gate_up, torch.cat([t[p + "mlp.gate_proj.weight"][isl],
                                                            t[p + "mlp.up_proj.weight"][isl]]))
                assert torch.equal(lw.w_down, t[p + "mlp.down_proj.weight"][:, isl])
                assert torch.equal(lw.q_norm, t[p + "self_attn.q_norm.weight"])
                assert torch.equal(lw.ln2, t[p + "post_attention_layernorm.weight"])
            assert torch.equal(w.lm_head, t["lm_head.weight"])
            assert torch.equal(w.embed, t["model.embed_tokens.weight"])


def test_missing_tensor_is_reported(tmp_path):
    from safetensors.torch import save_file

    from vllm_b200.model.hf_loader import load_hf_weights
    t = _tensors()
    del t["model.layers.1.mlp.up_proj.weight"]
    save_file(t, str(tmp_path / "model.safetensors"))
    with open(tmp_path / "config.json", "w") as f:
        json.dump(CFG, f)
    with pytest.raises(KeyError, match="up_proj"):
        load_hf_weights(str(tmp_path), torch.device("cpu"))
