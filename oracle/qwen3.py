"""Oracle Qwen3 forward + greedy loop for small configs (test infrastructure only).

Restates vllm-jax's model dataflow (vllm/model/qwen3.py) on the reference's
default path (Pallas kernels, USE_*_KERNEL = True):
  :432-444  embed -> layers -> final norm;   :474-477  logits = x @ lm_head
  :375-389  h = norm(x); attn; x = x + attn (bf16); h = norm(x); mlp; x = x + mlp
  :284-301  q/k/v = Einsum (fp32 accumulate, bf16 out); q_norm/k_norm; RoPE;
            attention(kv_cache, q, k, v); o_proj
  :337-341  SwiGLU: silu(gate) * up, bf16
  attention (:172-218): KV scatter, then
     prefill: q * bf16(1/sqrt(D)) in bf16 (prefill:60), fp32 logits, causal
              mask, softmax with P rounded to bf16 before PV (prefill:125-126)
     decode:  q / bf16(sqrt(D)) in bf16 (qwen3.py:207), fp32 logits, P in bf16
              (decode:116)
Each GEMM accumulates in fp32 (numpy) and rounds once to bf16; elementwise
ops round to bf16 after each jnp op. Weights come in as float32 arrays of
bf16 values.
"""
from __future__ import annotations

import numpy as np

from . import kv_store as okv
from .attention import gather_pages
from .bf16 import bf16


def _mm(x, w):
    """bf16(x @ w.T) with fp32 accumulation; w is [out, in]."""
    return bf16(np.matmul(x.astype(np.float32), w.T.astype(np.float32)))


def _silu(x):
    return bf16(x / (1.0 + np.exp(-x.astype(np.float64))).astype(np.float32))


def _softmax_pv(scores, v, mask):
    """fp32 scores [..., L] (masked -inf) -> P in bf16 -> fp32 PV -> normalised."""
    s = np.where(mask, scores, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    pb = bf16(p)
    return np.matmul(pb, v) / l


class OracleQwen3:
    """cfg: vllm_b200 Qwen3Config-like object; W: dict from Qwen3Weights.full_numpy()."""

    def __init__(self, cfg, W, num_blocks: int, block_size: int):
        self.cfg, self.W = cfg, W
        self.bs = block_size
        Hkv, D = cfg.num_key_value_heads, cfg.head_dim
        self.kc = [np.zeros((num_blocks, block_size, Hkv, D), np.float32)
                   for _ in range(cfg.num_hidden_layers)]
        self.vc = [np.zeros_like(self.kc[0]) for _ in range(cfg.num_hidden_layers)]

    def _layer(self, l, x, positions, slots, attn):
        c, lw = self.cfg, self.W["layers"][l]
        T = x.shape[0]
        Hq, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        h = okv.rmsnorm(x, lw["ln1"], c.rms_norm_eps)
        qkv = _mm(h, lw["w_qkv"])
        q = qkv[:, :Hq * D].reshape(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
        q, _ = okv.kv_store_qknorm_rope(q, k, v, lw["q_norm"], lw["k_norm"], positions, slots,
                                        self.kc[l], self.vc[l], eps=c.rms_norm_eps,
                                        rope_theta=c.rope_theta)
        o = attn(l, q).reshape(T, Hq * D)
        x = bf16(x + _mm(o, lw["w_o"]))
        h = okv.rmsnorm(x, lw["ln2"], c.rms_norm_eps)
        gu = _mm(h, lw["w_gate_up"])
        I = gu.shape[1] // 2
        m = bf16(_silu(gu[:, :I]) * gu[:, I:])
        return bf16(x + _mm(m, lw["w_down"]))

    def prefill(self, ids, positions, slots, cu, num_seqs):
        x = bf16(self.W["embed"][np.asarray(ids)])
        return self.prefill_layers(x, positions, slots, cu, num_seqs)

    def prefill_layers(self, x, positions, slots, cu, num_seqs, layers=None):
        """The decoder layers of a packed prefill on hidden states x [T, hidden]."""
        c = self.cfg
        D = c.head_dim
        g = c.num_attention_heads // c.num_key_value_heads
        qscale = float(bf16(np.float32(1.0 / np.sqrt(D))))

        def attn(l, q):
            out = np.zeros_like(q)
            qs = bf16(q * np.float32(qscale))
            for s in range(num_seqs):
                a, b = int(cu[s]), int(cu[s + 1])
                n = b - a
                sl = np.asarray(slots[a:b])
                flat_k = self.kc[l].reshape(-1, *self.kc[l].shape[2:])
                flat_v = self.vc[l].reshape(-1, *self.vc[l].shape[2:])
                k = flat_k[sl].transpose(1, 0, 2)            # [Hkv, n, D]
                v = flat_v[sl].transpose(1, 0, 2)
                qh = qs[a:b].reshape(n, -1, g, D).transpose(1, 2, 0, 3)   # [Hkv, g, n, D]
                sc = np.matmul(qh, k[:, None].transpose(0, 1, 3, 2))     # [Hkv, g, n, n]
                mask = np.tril(np.ones((n, n), bool))[None, None]
                o = _softmax_pv(sc, v[:, None], mask)                     # [Hkv, g, n, D]
                out[a:b] = bf16(o.transpose(2, 0, 1, 3).reshape(n, -1, D))
            return out

        for l in range(c.num_hidden_layers if layers is None else layers):
            x = self._layer(l, x, positions, slots, attn)
        return x

    def decode(self, ids, positions, slots, block_tables, ctx):
        c = self.cfg
        x = bf16(self.W["embed"][np.asarray(ids)])
        x = self.decode_layers(x, positions, slots, block_tables, ctx)
        x = okv.rmsnorm(x, self.W["norm"], c.rms_norm_eps)
        return _mm(x, self.W["lm_head"])

    def decode_layers(self, x, positions, slots, block_tables, ctx, layers=None):
        """The decoder layers of a decode step on hidden states x [B, hidden]
        (all layers, or the first `layers`)."""
        c = self.cfg
        D = c.head_dim
        g = c.num_attention_heads // c.num_key_value_heads
        sq = np.float32(bf16(np.float32(np.sqrt(np.float32(D)))))

        def attn(l, q):
            out = np.zeros_like(q)
            qs = bf16(q / sq)
            for b, L in enumerate(ctx):
                if L <= 0:
                    continue
                k = gather_pages(self.kc[l], block_tables[b], L).transpose(1, 0, 2)
                v = gather_pages(self.vc[l], block_tables[b], L).transpose(1, 0, 2)
                qh = qs[b].reshape(-1, g, D)                              # [Hkv, g, D]
                sc = np.matmul(qh, k.transpose(0, 2, 1))                  # [Hkv, g, L]
                o = _softmax_pv(sc, v, np.ones_like(sc, bool))
                out[b] = bf16(o.reshape(-1, D))
            return out

        for l in range(c.num_hidden_layers if layers is None else layers):
            x = self._layer(l, x, positions, slots, attn)
        return x


def _mixed_attn(model, starts, ns, tables):
    """Attention of a chunked step: new token i of sequence s sits at position
    starts[s] + i and attends to the cached keys [0, starts[s] + i] read
    through its block table. One-token rows scale q like the reference's
    decode (q / bf16(sqrt(D))), longer rows like its prefill (q * bf16(1/sqrt(D)))."""
    c = model.cfg
    D = c.head_dim
    g = c.num_attention_heads // c.num_key_value_heads
    sq = np.float32(bf16(np.float32(np.sqrt(np.float32(D)))))
    qscale = np.float32(bf16(np.float32(1.0 / np.sqrt(D))))

    def attn(l, q):
        out = np.zeros_like(q)
        a = 0
        for s, (st, n) in enumerate(zip(starts, ns)):
            L = st + n
            k = gather_pages(model.kc[l], tables[s], L).transpose(1, 0, 2)   # [Hkv, L, D]
            v = gather_pages(model.vc[l], tables[s], L).transpose(1, 0, 2)
            qs = bf16(q[a:a + n] / sq) if n == 1 else bf16(q[a:a + n] * qscale)
            qh = qs.reshape(n, -1, g, D).transpose(1, 2, 0, 3)               # [Hkv, g, n, D]
            sc = np.matmul(qh, k[:, None].transpose(0, 1, 3, 2))             # [Hkv, g, n, L]
            mask = (np.arange(L)[None, :] <= (st + np.arange(n))[:, None])[None, None]
            o = _softmax_pv(sc, v[:, None], mask)
            out[a:a + n] = bf16(o.transpose(2, 0, 1, 3).reshape(n, -1, D))
            a += n
        return out
    return attn


def mixed_step(model: OracleQwen3, ids, starts, ns, tables, sample_rows):
    """One chunked-prefill forward (tokens packed in sequence order, no
    padding); returns logits [len(sample_rows), vocab]."""
    c, bs = model.cfg, model.bs
    pos, slots = [], []
    for st, n, tb in zip(starts, ns, tables):
        for t in range(st, st + n):
            pos.append(t)
            slots.append(int(tb[t // bs]) * bs + t % bs)
    attn = _mixed_attn(model, starts, ns, tables)
    x = bf16(model.W["embed"][np.asarray(ids)])
    for l in range(c.num_hidden_layers):
        x = model._layer(l, x, pos, slots, attn)
    x = okv.rmsnorm(x[np.asarray(sample_rows, np.int64)], model.W["norm"], c.rms_norm_eps)
    return _mm(x, model.W["lm_head"])


def greedy_replay_chunked(model: OracleQwen3, trace: list, prompts: list[list[int]],
                          first_id: int = 0):
    """Replay a recorded chunked schedule (per step: (request id, start, n)
    and each request's block ids) with the oracle's own tokens. Returns
    (tokens per request index, per step a dict request index -> (top id, top
    logit, top-2 gap))."""
    tokens = {i: list(p) for i, p in enumerate(prompts)}
    gaps = []
    for st in trace:
        rows = [(rid - first_id, a, n) for rid, a, n in st["batch"]]
        ids, starts, ns, tables, sample, picked = [], [], [], [], [], []
        off = 0
        for (r, a, n), (rid, _, _) in zip(rows, st["batch"]):
            ids.extend(tokens[r][a:a + n])
            starts.append(a)
            ns.append(n)
            tables.append(np.asarray(st["blocks"][rid]))
            off += n
            if a + n == len(tokens[r]):
                sample.append(off - 1)
                picked.append(r)
        logits = mixed_step(model, ids, starts, ns, tables, sample)
        step = {}
        for row, r in enumerate(picked):
            lg = logits[row]
            top = int(np.argmax(lg))
            srt = np.sort(lg)
            step[r] = (top, float(srt[-1]), float(srt[-1] - srt[-2]))
            tokens[r].append(top)
        gaps.append(step)
    return tokens, gaps


def greedy_replay(model: OracleQwen3, trace: dict, prompts: list[list[int]],
                  forced: dict[int, list[int]] | list[list[int]] | None = None):
    """Replay the scheduled steps of a golden host trace (block tables, slots
    and positions depend only on lengths there). Without `forced` the oracle
    feeds back its own argmax; with `forced` (completion tokens per request,
    e.g. another engine's output) it feeds those instead, so every step of
    that engine can be checked against the oracle's logits for the same
    history. Returns (tokens per request id, per decode step a list of (top
    id, top logit, top-2 logit gap, logit of the token fed back) per
    scheduled row)."""
    tokens = {i: list(p) for i, p in enumerate(prompts)}
    gaps = []
    for st in trace["steps"]:
        if "decode" in st:
            d = st["decode"]
            ids = [tokens[r][-1] for r in st["decode_ids"]]
            ids += [0] * (len(d["input_ids"]) - len(ids))
            logits = model.decode(ids, d["positions"], d["slot_mapping"],
                                  np.asarray(d["block_tables"]), d["context_lens"])
            step = []
            for row, r in enumerate(st["decode_ids"]):
                lg = logits[row]
                top = int(np.argmax(lg))
                srt = np.sort(lg)
                nxt = top
                if forced is not None:
                    nxt = int(forced[r][len(tokens[r]) - len(prompts[r])])
                step.append((top, float(srt[-1]), float(srt[-1] - srt[-2]), float(lg[nxt])))
                tokens[r].append(nxt)
            gaps.append(step)
        if "prefill" in st:
            p = st["prefill"]
            ids = []
            for r in st["prefill_ids"]:
                ids.extend(tokens[r])
            ids += [0] * (len(p["input_ids"]) - len(ids))
            model.prefill(ids, p["positions"], p["slot_mapping"], p["cu_seqlens_q"],
                          len(st["prefill_ids"]))
    return tokens, gaps
