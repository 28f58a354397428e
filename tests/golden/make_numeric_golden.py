"""Generate numeric golden fixtures by running the reference's OWN attention,
RoPE and KV-scatter code -- TEST INFRASTRUCTURE.

Loads, from the vllm-jax checkout named by $VLLM_JAX_REF (or argv[1]), the
unmodified files
  vllm/kernels/decode_paged_attention.py   (Pallas decode kernel + combine,
                                            paged_attention_reference)
  vllm/kernels/prefill_paged_attention.py  (Pallas prefill kernel + merge,
                                            prefill_paged_attention_reference)
  vllm/model/qwen3.py                      (apply_rope, _update_kv_cache,
                                            attention(), _decode_attention,
                                            _prefill_attention)
with `jax` replaced by tests/golden/jax_shim.py (numpy + ml_dtypes with
JAX's dtype rules and a Pallas interpreter) and flax / transformers by empty
stubs (no flax layer is called here). Inputs come from det_inputs.py; only
outputs are written, to tests/golden/numerics.npz (bf16 bit patterns as
uint16).

Scenarios (shapes at the C1 config's heads: 16 q heads, 8 KV heads, d 128):
  rope          apply_rope(x, positions, 128, 1e6, None) at positions up to
                2^20 (bf16 position rounding above 256)
  kv_update     _update_kv_cache with slots -1 / -3 (wrap), 64 / 200 / -65 (drop)
  decode_*      attention() with DecodeAttentionMetadata: the default path
                (q / bf16(sqrt(128)), Pallas kernel, k_splits 16, combine),
                the jnp path (_decode_attention), and
                paged_attention_reference on the gathered K/V
  prefill_*     attention() with PrefillAttentionMetadata (17/30/45 tokens
                packed into a 128-token bucket): the jnp path
                (_prefill_attention), prefill_paged_attention_reference, and
                the Pallas kernel's first q block of every sequence (rows
                0..15), see `pallas_prefill_rows_beyond_first_block` below

Run:  VLLM_JAX_REF=<vllm-jax checkout> python tests/golden/make_numeric_golden.py
"""
from __future__ import annotations

import dataclasses
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

import det_inputs as di          # noqa: E402
import jax_shim                  # noqa: E402

REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VLLM_JAX_REF", "."))
OUT = HERE / "numerics.npz"


def _stubs():
    flax = types.ModuleType("flax")
    nnx = types.SimpleNamespace(
        Module=object, jit=lambda f: f, initializers=types.SimpleNamespace(uniform=lambda: None),
        with_partitioning=lambda f, spec: f, Einsum=None, RMSNorm=None, Linear=None, Embed=None,
        Rngs=None, List=list, Param=None)
    struct = types.SimpleNamespace(
        dataclass=dataclasses.dataclass,
        field=lambda pytree_node=True, **kw: dataclasses.field(**kw))
    flax.nnx, flax.struct = nnx, struct
    transformers = types.ModuleType("transformers")
    transformers.Qwen3Config = object
    transformers.modeling_flax_utils = types.SimpleNamespace(ACT2FN={})
    sys.modules["flax"] = flax
    sys.modules["transformers"] = transformers


def _load(name: str, rel: str):
    spec = importlib.util.spec_from_file_location(name, REF / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_reference():
    jax_shim.install()
    _stubs()
    for name in ("vllm", "vllm.kernels", "vllm.model"):
        pkg = types.ModuleType(name)
        pkg.__path__ = []
        sys.modules[name] = pkg
    ref = types.SimpleNamespace()
    ref.decode = _load("vllm.kernels.decode_paged_attention",
                       "vllm/kernels/decode_paged_attention.py")
    ref.prefill = _load("vllm.kernels.prefill_paged_attention",
                        "vllm/kernels/prefill_paged_attention.py")
    ref.qwen3 = _load("vllm.model.qwen3", "vllm/model/qwen3.py")
    return ref


J = jax_shim.bf16_array


def bits(x) -> np.ndarray:
    return np.asarray(x).astype(jax_shim.BF16).view(np.uint16)


def _i32(x):
    return jax_shim.wrap(np.asarray(x, np.int32))


def run_rope(ref):
    x, pos = di.rope_inputs()
    return ref.qwen3.apply_rope(J(x), _i32(pos), 128, 1_000_000.0, None)


def run_kv_update(ref):
    cache, slots, k, v = di.kv_update_inputs()
    return ref.qwen3._update_kv_cache(J(cache), _i32(slots), J(k), J(v))


def run_decode(ref):
    d = di.decode_inputs()
    q3 = ref.qwen3
    meta = q3.DecodeAttentionMetadata(input_positions=_i32(d["positions"]),
                                      slot_mapping=_i32(d["slot_mapping"]),
                                      block_tables=_i32(d["block_tables"]),
                                      context_lens=_i32(d["context_lens"]))
    out = {}
    q3.USE_DECODE_PAGED_ATTENTION_KERNEL = True
    kv_after, out["decode_pallas"] = q3.attention(J(d["kv_cache"]), J(d["q"]), J(d["k"]),
                                                  J(d["v"]), meta)
    q3.USE_DECODE_PAGED_ATTENTION_KERNEL = False
    _, out["decode_jnp"] = q3.attention(J(d["kv_cache"]), J(d["q"]), J(d["k"]), J(d["v"]), meta)
    # paged_attention_reference on the K/V gathered through the block tables,
    # with the dispatcher's q scaling (qwen3.py:207)
    bs, W = di.C1_HEADS["block_size"], di.C1_HEADS["width"]
    flat = np.asarray(kv_after).reshape(2, -1, *np.shape(kv_after)[-2:])
    bt = np.where(d["block_tables"] >= 0, d["block_tables"], 0)
    slots = (bt[:, :, None] * bs + np.arange(bs)[None, None]).reshape(len(bt), W * bs)
    kg, vg = flat[0][slots], flat[1][slots]                    # [B, W*bs, Hkv, D]
    q = J(d["q"])
    jnp = sys.modules["jax.numpy"]
    q_scaled = q / jnp.sqrt(jnp.asarray(q.shape[-1], dtype=q.dtype))
    out["decode_refimpl"] = ref.decode.paged_attention_reference(
        q_scaled, jax_shim.wrap(kg), jax_shim.wrap(vg), _i32(d["context_lens"]))
    # the scatter touched exactly the wrapped slots of the new tokens; keep those
    before = np.asarray(J(d["kv_cache"])).reshape(flat.shape)
    wrapped = np.where(d["slot_mapping"] < 0, d["slot_mapping"] + flat.shape[1],
                       d["slot_mapping"])
    untouched = np.ones(flat.shape[1], bool)
    untouched[wrapped] = False
    assert np.array_equal(bits(flat[:, untouched]), bits(before[:, untouched]))
    out["decode_kv_written"] = flat[:, wrapped]
    out["decode_kv_written_slots"] = wrapped.astype(np.int32)
    return out


def run_prefill(ref):
    d = di.prefill_inputs()
    q3 = ref.qwen3
    cu = _i32(d["cu_seqlens"])
    meta = q3.PrefillAttentionMetadata(
        input_positions=_i32(d["positions"]), slot_mapping=_i32(d["slot_mapping"]),
        block_tables=_i32(d["block_tables"]), cu_seqlens_q=cu, cu_seqlens_k=cu,
        max_seqlen_q=_i32(max(di.PREFILL_LENS)), max_seqlen_k=_i32(max(di.PREFILL_LENS)),
        max_seqlen_bucket=d["max_seqlen_bucket"])
    out = {}
    q3.USE_PREFILL_PAGED_ATTENTION_KERNEL = False
    kv_after, out["prefill_jnp"] = q3.attention(J(d["kv_cache"]), J(d["q"]), J(d["k"]),
                                                J(d["v"]), meta)
    q3.USE_PREFILL_PAGED_ATTENTION_KERNEL = True
    _, pallas = q3.attention(J(d["kv_cache"]), J(d["q"]), J(d["k"]), J(d["v"]), meta)
    k_pages = jax_shim.wrap(np.transpose(np.asarray(kv_after)[0], (2, 0, 1, 3)))
    v_pages = jax_shim.wrap(np.transpose(np.asarray(kv_after)[1], (2, 0, 1, 3)))
    out["prefill_refimpl"] = ref.prefill.prefill_paged_attention_reference(
        J(d["q"]), k_pages, v_pages, _i32(d["block_tables"]), cu, _i32(d["slot_mapping"]),
        _i32(d["positions"]), max_seqlen_bucket=d["max_seqlen_bucket"])
    # The Pallas kernel's q BlockSpec index_map returns qblock * block_m for a
    # Blocked dimension of size block_m (prefill_paged_attention.py:301-309),
    # i.e. an element offset where Pallas takes a block index: q blocks after
    # the first read rows qblock * block_m^2 (clamped). Rows 0..15 of each
    # sequence are unaffected; those are kept as a fixture.
    first = np.zeros(d["q"].shape[0], bool)
    for s, L in enumerate(di.PREFILL_LENS):
        a = int(d["cu_seqlens"][s])
        first[a:a + min(L, 16)] = True
    out["prefill_pallas_first_block"] = np.where(first[:, None, None], np.asarray(pallas), 0)
    out["prefill_first_block_rows"] = first
    pal = np.asarray(pallas).astype(np.float32)
    jn = np.asarray(out["prefill_jnp"]).astype(np.float32)
    rest = ~first[:d["num_tokens"]]
    out["pallas_prefill_rows_beyond_first_block_maxdiff"] = np.float32(
        np.abs(pal[:d["num_tokens"]][rest] - jn[:d["num_tokens"]][rest]).max())
    out["pallas_prefill_first_block_maxdiff"] = np.float32(
        np.abs(pal[first] - jn[first]).max())
    return out


def main():
    ref = load_reference()
    res = {"rope": run_rope(ref), "kv_update": run_kv_update(ref)}
    res.update(run_decode(ref))
    res.update(run_prefill(ref))
    store = {}
    for k, v in res.items():
        a = np.asarray(v)
        store[k] = bits(a) if a.dtype == jax_shim.BF16 else a
    np.savez_compressed(OUT, **store)
    for k, v in sorted(store.items()):
        print(f"{k:48s} {v.dtype} {v.shape}" + (f" = {float(v)}" if v.ndim == 0 else ""))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
