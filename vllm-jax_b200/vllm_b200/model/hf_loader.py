"""Qwen3 checkpoints in the Hugging Face layout (safetensors), sharded for TP.

Counterpart of vllm-jax's vllm/utils/hf_convert.py:30-198, which maps HF
names onto the flax model (transposing every projection for `x @ kernel`).
Here the projections stay in HF's [out, in] layout, which is what the
engine's `F.linear` / `x @ w.T` GEMMs want, and are fused and sliced per
rank: q/k/v rows of this rank's KV heads (and their query heads) are
concatenated into w_qkv, gate/up rows of its intermediate slice into
w_gate_up, and the columns of o_proj / down_proj are sliced to match. Names
and the tied lm_head follow hf_convert.py:70-108 and :164-165; single files
and `model.safetensors.index.json` shards are read as at :117-154, lazily,
one tensor at a time (`safe_open`), so a rank only materialises its slices.
No download: `path` must be a local directory (or file).
"""
from __future__ import annotations

import json
import os

import torch

from .qwen3 import LayerWeights, Qwen3Config, Qwen3Weights


def config_from_hf(path: str) -> Qwen3Config:
    """Qwen3Config from a checkpoint directory's config.json."""
    with open(os.path.join(path, "config.json"), encoding="utf-8") as f:
        c = json.load(f)
    theta = c.get("rope_theta")
    if theta is None:  # transformers >= 5 moves it into rope_parameters
        theta = (c.get("rope_parameters") or {}).get("rope_theta", 1_000_000.0)
    heads = c["num_attention_heads"]
    return Qwen3Config(vocab_size=c["vocab_size"], hidden_size=c["hidden_size"],
                       intermediate_size=c["intermediate_size"],
                       num_hidden_layers=c["num_hidden_layers"], num_attention_heads=heads,
                       num_key_value_heads=c.get("num_key_value_heads", heads),
                       head_dim=c.get("head_dim", c["hidden_size"] // heads),
                       rms_norm_eps=c.get("rms_norm_eps", 1e-6), rope_theta=float(theta),
                       tie_word_embeddings=c.get("tie_word_embeddings", False))


def _tensor_files(path: str) -> dict[str, str]:
    """HF tensor name -> safetensors file holding it."""
    from safetensors import safe_open
    if os.path.isfile(path):
        files = [path]
    else:
        single = os.path.join(path, "model.safetensors")
        index = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(single):
            files = [single]
        elif os.path.exists(index):
            with open(index, encoding="utf-8") as f:
                wm = json.load(f)["weight_map"]
            return {k: os.path.join(path, v) for k, v in wm.items()}
        else:
            raise FileNotFoundError(f"no model.safetensors or index under {path}")
    out = {}
    for fn in files:
        with safe_open(fn, framework="pt") as f:
            for k in f.keys():
                out[k] = fn
    return out


class _Reader:
    def __init__(self, path: str):
        from safetensors import safe_open
        self._safe_open = safe_open
        self.where = _tensor_files(path)
        self._open: dict[str, object] = {}

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name}")
        fn = self.where[name]
        if fn not in self._open:
            self._open[fn] = self._safe_open(fn, framework="pt")
        return self._open[fn].get_tensor(name)


def load_hf_weights(path: str, device: torch.device, tp_rank: int = 0, tp_size: int = 1,
                    cfg: Qwen3Config | None = None) -> Qwen3Weights:
    """Qwen3Weights of rank `tp_rank` of `tp_size` from a local HF checkpoint."""
    cfg = cfg or config_from_hf(path)
    H, D, I = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if Hkv % tp_size or I % tp_size:
        raise ValueError(f"tensor_parallel_size {tp_size} must divide {Hkv} KV heads and "
                         f"intermediate {I}")
    hq_l, hkv_l, i_l = Hq // tp_size, Hkv // tp_size, I // tp_size
    r = tp_rank
    qs = slice(r * hq_l * D, (r + 1) * hq_l * D)
    ks = slice(r * hkv_l * D, (r + 1) * hkv_l * D)
    isl = slice(r * i_l, (r + 1) * i_l)
    rd = _Reader(path)
    bf = lambda t: t.to(torch.bfloat16)
    dev = lambda t: bf(t).to(device).contiguous()

    w = object.__new__(Qwen3Weights)
    w.cfg, w.tp_rank, w.tp_size = cfg, tp_rank, tp_size
    w.embed = dev(rd.get("model.embed_tokens.weight"))
    w.layers = []
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        g = lambda n: rd.get(p + n)
        wq, wk, wv = g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"), \
            g("self_attn.v_proj.weight")
        if wq.shape != (Hq * D, H) or wk.shape != (Hkv * D, H):
            raise ValueError(f"layer {l}: q/k projection shapes {tuple(wq.shape)}, "
                             f"{tuple(wk.shape)} do not match the config")
        w.layers.append(LayerWeights(
            w_qkv=dev(torch.cat([bf(wq[qs]), bf(wk[ks]), bf(wv[ks])])),
            w_o=dev(g("self_attn.o_proj.weight")[:, qs]),
            w_gate_up=dev(torch.cat([bf(g("mlp.gate_proj.weight")[isl]),
                                     bf(g("mlp.up_proj.weight")[isl])])),
            w_down=dev(g("mlp.down_proj.weight")[:, isl]),
            ln1=dev(g("input_layernorm.weight")), ln2=dev(g("post_attention_layernorm.weight")),
            q_norm=dev(g("self_attn.q_norm.weight")), k_norm=dev(g("self_attn.k_norm.weight"))))
    w.norm = dev(rd.get("model.norm.weight"))
    if cfg.tie_word_embeddings or "lm_head.weight" not in rd:
        w.lm_head = w.embed
    else:
        w.lm_head = dev(rd.get("lm_head.weight"))
    return w
