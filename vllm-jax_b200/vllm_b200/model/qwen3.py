"""Qwen3 decoder in torch around the sm_100a attention path.

Dataflow per layer follows vllm-jax's vllm/model/qwen3.py:375-389
(Qwen3DecoderLayer): input RMSNorm -> q/k/v projections -> per-head q/k
RMSNorm -> RoPE -> KV store -> paged attention -> o_proj -> residual add ->
post-attention RMSNorm -> SwiGLU MLP -> residual add; then the final norm and
the (tied or untied) lm_head (:474-477). What changes:
  * q/k norm, RoPE and the KV-slot scatter are one kernel (K3), prefill and
    decode attention are K1 / K2 (libvjattn); dense GEMMs are cuBLAS.
  * tensor parallelism by KV head: rank r holds q/k/v heads of KV heads
    [r*Hkv/t, (r+1)*Hkv/t), the matching o_proj columns, 1/t of the MLP, and
    one NCCL all-reduce follows o_proj and one follows down_proj (the
    reference's Mesh annotations at qwen3.py:245-332 describe the same split).
`attention(kv_cache, q, k, v, metadata)` keeps the reference boundary
(qwen3.py:172-218) for callers that run their own projections.

Weights are random (BASELINE: N(0, 0.02), seed 0): each tensor is drawn in a
fixed order from a generator seeded with (seed, layer, name) and sliced for
the rank, so every TP degree sees the same full model. RMSNorm scales are 1.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..kernels.decode_paged_attention import paged_decode
from ..kernels.fused import add_rmsnorm, silu_mul
from ..kernels.gemm import TiledWeight, decode_gemm, gemm_workspace_bytes, qkv_gemm_kv_store
from ..kernels.kv_store import kv_store_qknorm_rope
from ..kernels.prefill_paged_attention import paged_attention_mixed, paged_prefill


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = True


PRESETS = {
    "Qwen3-0.6B": Qwen3Config(),
    "Qwen3-8B": Qwen3Config(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                            num_attention_heads=32, tie_word_embeddings=False),
    "Qwen3-32B": Qwen3Config(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                             num_attention_heads=64, tie_word_embeddings=False),
}


def get_config(name: str) -> Qwen3Config:
    key = name.split("/")[-1]
    if key not in PRESETS:
        raise ValueError(f"unknown model {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]


# ---------------------------------------------------------------------------
# metadata structs of the attention boundary (vllm/model/qwen3.py:17-37)
# ---------------------------------------------------------------------------
@dataclass
class DecodeAttentionMetadata:
    input_positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor


@dataclass
class PrefillAttentionMetadata:
    input_positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    cu_seqlens_q: torch.Tensor
    cu_seqlens_k: torch.Tensor
    max_seqlen_q: int
    max_seqlen_k: int
    max_seqlen_bucket: int
    num_seqs: int | None = None          # sequences actually present (<= rows of block_tables)
    context_lens: torch.Tensor | None = None  # keys per sequence (cached prefix + new)


def attention(kv_cache: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              metadata) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for vllm/model/qwen3.py:172-218: store k/v (in place), then paged
    prefill or decode attention. Returns (kv_cache, out [T, Hq, D]).

    q is scaled the reference's way, in bf16, by the same launch that stores
    k/v: decode divides by bf16(sqrt(D)) (qwen3.py:207), prefill multiplies
    by bf16(1/sqrt(D)) (prefill_paged_attention.py:60); attention then runs
    with scale 1."""
    prefill = isinstance(metadata, PrefillAttentionMetadata)
    qs = kv_store_qknorm_rope(q, k, v, kv_cache, metadata.slot_mapping, norm=False, rope=False,
                              q_scale="mul" if prefill else "div")
    if prefill:
        S = metadata.num_seqs if metadata.num_seqs is not None else metadata.block_tables.shape[0]
        out = paged_prefill(qs, kv_cache, metadata.block_tables[:S],
                            metadata.cu_seqlens_q[:S + 1], metadata.context_lens,
                            max_seqlen_q=metadata.max_seqlen_bucket, scale=1.0)
    else:
        out = paged_decode(qs, kv_cache, metadata.block_tables, metadata.context_lens, 1.0)
    return kv_cache, out


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------
def _draw(shape, seed: int, tag: int, gen_device: str, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator(device=gen_device)
    g.manual_seed((seed * 1_000_003 + tag) & 0x7FFFFFFFFFFFFFFF)
    return (torch.randn(shape, generator=g, device=gen_device, dtype=torch.float32) * std).to(
        torch.bfloat16)


@dataclass
class LayerWeights:
    w_qkv: torch.Tensor     # [(Hq_l + 2 Hkv_l) * D, hidden]
    w_o: torch.Tensor       # [hidden, Hq_l * D]
    w_gate_up: torch.Tensor  # [2 * I_l, hidden]
    w_down: torch.Tensor    # [hidden, I_l]
    ln1: torch.Tensor
    ln2: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


class Qwen3Weights:
    """Random-init weights, sharded for (tp_rank, tp_size). Parameter order and
    the per-tensor seeds are fixed, so the full model is the same at every TP
    degree and on every generator device of the same kind."""

    def __init__(self, cfg: Qwen3Config, device: torch.device, seed: int = 0, tp_rank: int = 0,
                 tp_size: int = 1, gen_device: str | None = None):
        H, D, I = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
        Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        if Hkv % tp_size or I % tp_size:
            raise ValueError(f"tensor_parallel_size {tp_size} must divide {Hkv} KV heads and "
                             f"intermediate {I}")
        gen = gen_device or ("cuda" if device.type == "cuda" else "cpu")
        hq_l, hkv_l, i_l = Hq // tp_size, Hkv // tp_size, I // tp_size
        r = tp_rank
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        one = torch.ones(H, dtype=torch.bfloat16, device=device)
        oned = torch.ones(D, dtype=torch.bfloat16, device=device)
        self.embed = _draw((cfg.vocab_size, H), seed, 1, gen).to(device)
        self.layers: list[LayerWeights] = []
        for layer in range(cfg.num_hidden_layers):
            base = 100 + 16 * layer
            wq = _draw((Hq * D, H), seed, base + 0, gen)
            wk = _draw((Hkv * D, H), seed, base + 1, gen)
            wv = _draw((Hkv * D, H), seed, base + 2, gen)
            wo = _draw((H, Hq * D), seed, base + 3, gen)
            wg = _draw((I, H), seed, base + 4, gen)
            wu = _draw((I, H), seed, base + 5, gen)
            wd = _draw((H, I), seed, base + 6, gen)
            qs = slice(r * hq_l * D, (r + 1) * hq_l * D)
            ks = slice(r * hkv_l * D, (r + 1) * hkv_l * D)
            isl = slice(r * i_l, (r + 1) * i_l)
            self.layers.append(LayerWeights(
                w_qkv=torch.cat([wq[qs], wk[ks], wv[ks]]).to(device).contiguous(),
                w_o=wo[:, qs].to(device).contiguous(),
                w_gate_up=torch.cat([wg[isl], wu[isl]]).to(device).contiguous(),
                w_down=wd[:, isl].to(device).contiguous(),
                ln1=one, ln2=one, q_norm=oned, k_norm=oned))
            del wq, wk, wv, wo, wg, wu, wd
        self.norm = one
        self.lm_head = (self.embed if cfg.tie_word_embeddings
                        else _draw((cfg.vocab_size, H), seed, 2, gen).to(device))

    def pack_tiles(self) -> None:
        """Second copy of every projection weight packed for the decode GEMMs
        (vj_pack_weight_tiles: contiguous 16 KB swizzled tiles), kept beside
        the row-major weights that cuBLAS uses for prefill-sized batches.
        Costs one more copy of the projection weights in HBM."""
        if getattr(self, "tiles", None) is not None:
            return
        self.tiles = [dict(qkv=TiledWeight(lw.w_qkv), o=TiledWeight(lw.w_o),
                           gu=TiledWeight(lw.w_gate_up, "swiglu"), down=TiledWeight(lw.w_down))
                      for lw in self.layers]

    def full_numpy(self):
        """Every tensor as float32 numpy (unsharded models only; for the oracle)."""
        assert self.tp_size == 1
        f = lambda t: t.float().cpu().numpy()
        return {"embed": f(self.embed), "norm": f(self.norm), "lm_head": f(self.lm_head),
                "layers": [{k: f(getattr(lw, k)) for k in LayerWeights.__dataclass_fields__}
                           for lw in self.layers]}


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """flax RMSNorm semantics: fp32 statistics, bf16(x * (rsqrt(ms + eps) * w))."""
    xf = x.float()
    mul = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return (xf * mul).to(torch.bfloat16)


class Qwen3Model:
    """Forward passes of one rank. kv_caches[l]: (2, num_blocks, bs, Hkv_l, D) bf16."""

    def __init__(self, weights: Qwen3Weights, process_group=None, tp_comm=None,
                 reference_q_scaling: bool = False):
        self.w = weights
        self.cfg = weights.cfg
        self.pg = process_group
        # NVLink communicator (src/tp_comm.py): row-parallel GEMMs of up to
        # tp_comm.max_rows rows reduce through the fused peer-memory kernel
        self.tp_comm = tp_comm
        c = self.cfg
        self.hq = c.num_attention_heads // weights.tp_size
        self.hkv = c.num_key_value_heads // weights.tp_size
        self.d = c.head_dim
        self.scale = 1.0 / math.sqrt(c.head_dim)
        # reference_q_scaling: K3 scales q in bf16 like the reference (decode:
        # q / bf16(sqrt(D)), qwen3.py:207; prefill: q * bf16(1/sqrt(D)),
        # prefill_paged_attention.py:60) and attention runs with scale 1;
        # otherwise the attention kernels apply 1/sqrt(D) to q.k in fp32
        self.reference_q_scaling = reference_q_scaling
        # (cos, sin) table of K3 covering every position the engine can reach;
        # set by the model runner before any CUDA graph capture
        self.rope_table: torch.Tensor | None = None
        # split-KV scratch of the decode kernel, owned here so that captured
        # CUDA graphs keep a valid address (set by the model runner)
        self.decode_workspace: torch.Tensor | None = None
        # forwards of at most this many rows use the fused tcgen05 projections
        # (vj_qkv_gemm_kv_store, vj_decode_gemm); 0 = cuBLAS + separate kernels
        self.fused_gemm_rows = 0
        self.gemm_workspace: torch.Tensor | None = None

    def enable_fused_gemm(self, max_rows: int) -> None:
        """Use the fused projections for forwards of <= max_rows rows, with one
        zero-filled workspace sized for every row count up to max_rows
        (allocated here, before any CUDA graph capture, and never replaced)."""
        c, w = self.cfg, self.w
        w.pack_tiles()
        H, D = c.hidden_size, self.d
        I_l = w.layers[0].w_gate_up.shape[0] // 2
        shapes = ((w.layers[0].w_qkv.shape[0], H, "plain"), (H, self.hq * D, "plain"),
                  (2 * I_l, H, "swiglu"), (H, I_l, "plain"))
        need = 0
        for r in range(1, max_rows + 1):     # every row count: the split plan depends on it
            need = max([need] + [gemm_workspace_bytes(r, n, k, m) for n, k, m in shapes])
        self.gemm_workspace = torch.zeros(need, dtype=torch.uint8, device=w.layers[0].w_qkv.device)
        self.fused_gemm_rows = max_rows

    def _fused(self, T: int) -> bool:
        return 0 < T <= self.fused_gemm_rows and self.gemm_workspace is not None

    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.pg is not None and self.w.tp_size > 1:
            torch.distributed.all_reduce(x, group=self.pg)
        return x

    def _reduce_add_norm(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor,
                         w_norm: torch.Tensor, site: int, w_tiled: TiledWeight | None = None):
        """Row-parallel GEMM a @ w.T summed over ranks, added to the residual x,
        then RMSNorm: returns (new residual, normed). Under tensor parallelism
        the GEMM writes into the NVLink buffer and one kernel reduces, adds and
        normalises; otherwise NCCL all-reduce (or nothing) + vj_add_rmsnorm."""
        T = a.shape[0]
        eps = self.cfg.rms_norm_eps
        c = self.tp_comm
        fused = self._fused(T)
        if c is not None and T <= c.max_rows:
            if fused:
                decode_gemm(a, w_tiled or w, out=c.buffer(site, T), ws=self.gemm_workspace)
            else:
                torch.mm(a, w.t(), out=c.buffer(site, T))
            return c.allreduce_add_rmsnorm(site, T, x, w_norm, eps)
        d = decode_gemm(a, w_tiled or w, ws=self.gemm_workspace) if fused else F.linear(a, w)
        d = self._all_reduce(d)
        return add_rmsnorm(d, w_norm, eps, residual=x)

    def _layer(self, l: int, x: torch.Tensor, h: torch.Tensor, kv_cache: torch.Tensor, meta,
               attn_fn, w_next: torch.Tensor, q_scale: str | None):
        """x: residual stream entering layer l; h = input_layernorm(x). Returns
        (x after the layer, h = the next norm of it, with weight w_next)."""
        lw = self.w.layers[l]
        c = self.cfg
        T = x.shape[0]
        fused = self._fused(T)
        tw = self.w.tiles[l] if fused else None
        if fused:
            # qkv projection + q/k norm + RoPE + KV store in one launch
            q = qkv_gemm_kv_store(h, tw["qkv"], kv_cache, meta.slot_mapping, meta.positions,
                                  lw.q_norm, lw.k_norm, self.hq, eps=c.rms_norm_eps,
                                  rope_theta=c.rope_theta, q_scale=q_scale,
                                  table=self.rope_table, ws=self.gemm_workspace)
        else:
            qkv = F.linear(h, lw.w_qkv)
            q, k, v = torch.split(qkv, [self.hq * self.d, self.hkv * self.d, self.hkv * self.d],
                                  -1)
            q = kv_store_qknorm_rope(q.view(T, self.hq, self.d), k.view(T, self.hkv, self.d),
                                     v.view(T, self.hkv, self.d), kv_cache,
                                     meta.slot_mapping, meta.positions, lw.q_norm, lw.k_norm,
                                     eps=c.rms_norm_eps, rope_theta=c.rope_theta,
                                     q_scale=q_scale, table=self.rope_table)
        o = attn_fn(q, kv_cache).reshape(T, self.hq * self.d)
        # attn_output += x; post_attention_layernorm   (qwen3.py:375-389)
        x, h = self._reduce_add_norm(o, lw.w_o, x, lw.ln2, 0, tw and tw["o"])
        if fused:
            m = decode_gemm(h, tw["gu"], "swiglu", ws=self.gemm_workspace)
        else:
            m = silu_mul(F.linear(h, lw.w_gate_up))
        # outputs = residual + mlp; next input_layernorm (or the final norm)
        return self._reduce_add_norm(m, lw.w_down, x, w_next, 1, tw and tw["down"])

    def _stack(self, x: torch.Tensor, kv_caches, meta, attn_fn,
               q_scale: str | None = None) -> torch.Tensor:
        c = self.cfg
        L = c.num_hidden_layers
        h = add_rmsnorm(x, self.w.layers[0].ln1, c.rms_norm_eps)
        for l in range(L):
            w_next = self.w.layers[l + 1].ln1 if l + 1 < L else self.w.norm
            x, h = self._layer(l, x, h, kv_caches[l], meta, attn_fn, w_next, q_scale)
        return h    # final norm applied

    def _attn_scale(self, kind: str) -> tuple[str | None, float]:
        """(K3 q scaling, attention scale) of a prefill or decode forward."""
        if self.reference_q_scaling:
            return ("mul" if kind == "prefill" else "div"), 1.0
        return None, self.scale

    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(input_ids.long(), self.w.embed)

    def forward_prefill(self, meta, kv_caches: list[torch.Tensor]) -> torch.Tensor:
        """Packed prefill of meta.num_tokens tokens (bucket-padded); writes the
        KV caches and returns the final hidden states (the reference computes
        no logits in prefill, model_runner.py:41-59)."""
        x = self.embed(meta.input_ids)
        S = meta.num_seqs
        q_scale, scale = self._attn_scale("prefill")

        def attn(q, kv):
            return paged_prefill(q, kv, meta.block_tables[:S], meta.cu_seqlens_q[:S + 1],
                                 getattr(meta, "context_lens", None),
                                 max_seqlen_q=meta.max_seqlen_bucket, scale=scale)

        return self._stack(x, kv_caches, meta, attn, q_scale)

    def forward_decode(self, meta, kv_caches: list[torch.Tensor]) -> torch.Tensor:
        """One token per row; returns bf16 logits [rows, vocab]."""
        x = self.embed(meta.input_ids)
        planned = []   # the first layer plans the split; the others reuse it
        q_scale, scale = self._attn_scale("decode")

        def attn(q, kv):
            out = paged_decode(q, kv, meta.block_tables, meta.context_lens, scale,
                               workspace=self.decode_workspace,
                               reuse_plan=bool(planned) and self.decode_workspace is not None)
            planned.append(True)
            return out

        x = self._stack(x, kv_caches, meta, attn, q_scale)
        return F.linear(x, self.w.lm_head)           # compute_logits (qwen3.py:474-477)

    def forward_mixed(self, meta, kv_caches: list[torch.Tensor], num_decode: int,
                      sample_rows: torch.Tensor) -> torch.Tensor:
        """Chunked-prefill step over meta (ranges metadata): sequences
        [0, num_decode) contribute one token each, the rest are prompt chunks
        after a cached prefix; each layer's attention over both kinds is ONE
        kernel launch (vj_paged_attention_mixed: split-KV decode CTAs next to
        tcgen05 prefill CTAs), whose decode split plan the later layers reuse.
        Returns bf16 logits of `sample_rows`."""
        x = self.embed(meta.input_ids)
        S, nd = meta.num_seqs, num_decode

        planned = []

        def attn(q, kv):
            out = paged_attention_mixed(
                q, kv, meta.block_tables[:S], meta.cu_seqlens_q[:S + 1], meta.context_lens[:S],
                nd, meta.max_new, self.scale, workspace=self.decode_workspace,
                reuse_plan=bool(planned) and nd > 0 and self.decode_workspace is not None)
            planned.append(True)
            return out

        x = self._stack(x, kv_caches, meta, attn)
        return F.linear(x.index_select(0, sample_rows), self.w.lm_head)
