"""Oracle for token sampling (test infrastructure only).

Restates vllm/sampler.py:7-42 of vllm-jax on one logit row:
  :12-14  temperature <= 0 -> argmax (first index on ties)
  :16     x = logits / temperature, in the logits' dtype (bf16)
  :17-23  top_k > 0: lax.top_k keeps k values (equal values: lower index
          first); the rest become finfo.min
  :25-36  top_p < 1: stable argsort of -x; softmax; cumulative sum; keep
          cum <= top_p, and always the first sorted token
  :38-41  categorical draw (Gumbel-max in jax.random.categorical)
The softmax and cumulative sum are taken in float64 here; the reference
rounds them to bf16 (XLA's bf16 cumsum is not available to pin against), so
kept sets are compared away from ties with the top_p boundary (`margin`).
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16


def scaled(logits: np.ndarray, temperature: float) -> np.ndarray:
    """bf16(float32(logit) / float32(T)) with round-to-nearest-even."""
    return bf16(np.asarray(logits, np.float32) / np.float32(temperature))


def kept_mask(logits: np.ndarray, temperature: float, top_k: int, top_p: float):
    """Returns (kept mask over the vocab, x, margin): margin is the distance of
    the nearest cumulative probability to top_p (inf without top-p)."""
    x = scaled(logits, temperature)
    V = x.shape[0]
    order = np.lexsort((np.arange(V), -x.astype(np.float64)))
    keep = np.ones(V, bool)
    if 0 < top_k < V:
        keep = np.zeros(V, bool)
        keep[order[:top_k]] = True
    margin = np.inf
    if top_p < 1.0:
        xs = x[order].astype(np.float64)
        ks = keep[order]
        e = np.where(ks, np.exp(xs - xs[ks].max()), 0.0)
        cum = np.cumsum(e) / e.sum()
        km = (cum <= top_p) & ks
        km[0] = True
        margin = float(np.min(np.abs(cum[ks] - top_p)))
        keep = np.zeros(V, bool)
        keep[order[km]] = True
    return keep, x, margin


def probs(logits: np.ndarray, temperature: float, top_k: int, top_p: float) -> np.ndarray:
    """Sampling distribution: softmax(x) restricted to the kept set."""
    keep, x, _ = kept_mask(logits, temperature, top_k, top_p)
    xf = x.astype(np.float64)
    e = np.where(keep, np.exp(xf - xf[keep].max()), 0.0)
    return e / e.sum()
