"""A numpy + ml_dtypes stand-in for the slice of JAX that vllm-jax's numerics use
-- TEST INFRASTRUCTURE (fixture generation only).

jax / jaxlib / flax are not installable in this image, so the reference's own
attention, RoPE and KV-scatter code (vllm/model/qwen3.py, vllm/kernels/*.py)
is run here UNMODIFIED against this module, which is installed into
sys.modules as `jax`, `jax.numpy`, `jax.lax`, `jax.nn`,
`jax.experimental.pallas` (+ `.triton`) before the reference files are
loaded. What it emulates, and the JAX rule each piece follows:

* Arrays (`JArr`, an ndarray subclass) carry JAX's dtype rules: Python
  scalars are weakly typed (bf16_array * 0.5 stays bf16), strong dtypes
  promote on the lattice bool < int32 < bf16 < f32, every float op on bf16
  is computed in f32 and rounded once to bf16 (round-to-nearest-even, what
  XLA does for an unfused op), `sum` of bf16 accumulates in f32 and rounds
  once (jnp reductions upcast half types), comparisons give bool.
* `einsum` / `pl.dot`: f32 accumulation; the result has
  `preferred_element_type` if given (pl.dot: f32), else the inputs' type.
* `.at[idx].set(v, mode="drop")`: negative indices wrap once (JAX's
  `wrap_negative_indices=True` default), then out-of-range updates drop.
* `jax.nn.softmax`: exp(x - max) / sum, each op rounded in x's dtype.
* `pl.pallas_call` is an interpreter: the kernel runs once per grid point
  with refs that are numpy views of the blocks BlockSpecs select (Blocked
  indexing: index_map returns block indices, a `None` dim is squeezed and
  indexed by element), with start offsets clamped into the array as
  interpret mode's dynamic_slice does. `lax.fori_loop` / `lax.cond` run
  eagerly; `jax.vmap` loops over the mapped axis; `jax.jit` is the identity.

Known residual gap: XLA may fuse elementwise ops and keep f32 between them
(`xla_allow_excess_precision`); this shim rounds after every op, so single
bf16 ulps can differ from a real JAX run. Transcendentals use numpy's f32
implementations, not XLA's.
"""
from __future__ import annotations

import itertools
import math
import sys
import types

import ml_dtypes
import numpy as np

BF16 = np.dtype(ml_dtypes.bfloat16)
F32 = np.dtype(np.float32)
I32 = np.dtype(np.int32)
BOOL = np.dtype(np.bool_)
_RANK = {BOOL: 0, np.dtype(np.uint8): 1, np.dtype(np.int8): 1, np.dtype(np.int16): 1,
         I32: 2, np.dtype(np.int64): 2, np.dtype(np.uint32): 2, BF16: 3,
         np.dtype(np.float16): 3, F32: 4, np.dtype(np.float64): 4}


def _is_weak(x) -> bool:
    return isinstance(x, (bool, int, float)) and not isinstance(x, np.generic)


def _strong_dtype(x) -> np.dtype:
    return np.asarray(x).dtype


def result_dtype(*xs) -> np.dtype:
    """JAX promotion of the operands (Python scalars weak)."""
    strong = [_strong_dtype(x) for x in xs if not _is_weak(x)]
    weak = [x for x in xs if _is_weak(x)]
    if strong:
        dt = strong[0]
        for d in strong[1:]:
            if d == dt:
                continue
            if {d, dt} == {BF16, np.dtype(np.float16)}:
                dt = F32
            elif _RANK.get(d, 4) > _RANK.get(dt, 4):
                dt = d
        if dt.kind in "biu" and any(isinstance(w, float) for w in weak):
            return F32
        if dt.kind == "b" and any(isinstance(w, int) and not isinstance(w, bool) for w in weak):
            return I32
        if dt == np.dtype(np.float64):
            return F32
        if dt == np.dtype(np.int64):
            return I32
        return dt
    if any(isinstance(w, float) for w in weak):
        return F32
    if any(isinstance(w, int) and not isinstance(w, bool) for w in weak):
        return I32
    return BOOL


def _compute_dtype(dt: np.dtype) -> np.dtype:
    return F32 if dt.kind == "f" or dt == BF16 else dt


_COMPARE = {np.less, np.less_equal, np.greater, np.greater_equal, np.equal, np.not_equal}
_LOGICAL = {np.logical_and, np.logical_or, np.logical_not, np.logical_xor}
_BITWISE = {np.bitwise_and, np.bitwise_or, np.bitwise_xor, np.invert}


def wrap(x) -> "JArr":
    return np.asarray(x).view(JArr)


class _AtIndex:
    def __init__(self, arr, idx):
        self.arr, self.idx = arr, idx if isinstance(idx, tuple) else (idx,)

    def set(self, values, mode=None, **kw):
        out = np.array(self.arr, copy=True)
        comps = [np.asarray(c) if not isinstance(c, slice) else c for c in self.idx]
        if any(isinstance(c, slice) for c in comps):
            raise NotImplementedError("jax_shim .at[]: slices in a scatter index")
        lead = np.broadcast_arrays(*comps)
        norm = []
        valid = np.ones(lead[0].shape, bool)
        for d, c in enumerate(lead):
            c = c.astype(np.int64)
            c = np.where(c < 0, c + out.shape[d], c)           # wrap negative indices
            valid &= (c >= 0) & (c < out.shape[d])             # mode="drop"
            norm.append(c)
        vals = np.broadcast_to(np.asarray(values).astype(out.dtype),
                               lead[0].shape + out.shape[len(lead):])
        out[tuple(c[valid] for c in norm)] = vals[valid]
        return wrap(out)


class _At:
    def __init__(self, arr):
        self.arr = arr

    def __getitem__(self, idx):
        return _AtIndex(self.arr, idx)


class JArr(np.ndarray):
    """ndarray with JAX dtype semantics (see module docstring)."""

    @property
    def at(self):
        return _At(self)

    def __array_ufunc__(self, ufunc, method, *inputs, out=None, **kw):
        if out is not None:
            raise NotImplementedError("jax_shim: ufunc out=")
        if method == "__call__":
            return _call_ufunc(ufunc, inputs, kw)
        if method == "reduce":
            return _reduce(ufunc, inputs[0], kw)
        raise NotImplementedError(f"jax_shim: ufunc method {method}")

    def __bool__(self):
        return bool(np.asarray(self))

    def __index__(self):
        return int(np.asarray(self))

    def __int__(self):
        return int(np.asarray(self))

    def __float__(self):
        return float(np.asarray(self))


def _plain(x):
    return np.asarray(x).view(np.ndarray) if isinstance(x, np.ndarray) else x


def _call_ufunc(ufunc, inputs, kw):
    dt = result_dtype(*inputs)
    if ufunc in _COMPARE:
        cdt = _compute_dtype(dt)
        args = [np.asarray(_plain(x)).astype(dt).astype(cdt) for x in inputs]
        return wrap(ufunc(*args))
    if ufunc in _LOGICAL or ufunc in _BITWISE:
        args = [_plain(x) for x in inputs]
        return wrap(ufunc(*args).astype(dt if dt.kind != "f" else BOOL))
    cdt = _compute_dtype(dt)
    if ufunc is np.true_divide and cdt.kind in "iub":
        dt = cdt = F32
    # a weakly typed Python scalar takes the result dtype first (1e6 -> bf16 999424)
    args = [np.asarray(_plain(x)).astype(cdt) if not _is_weak(x) else
            np.asarray(x).astype(dt).astype(cdt) for x in inputs]
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        r = ufunc(*args)
    if dt.kind == "f" or dt == BF16:
        return wrap(np.asarray(r, cdt).astype(dt))
    return wrap(np.asarray(r).astype(dt))


def _reduce(ufunc, x, kw):
    a = np.asarray(_plain(x))
    axis = kw.get("axis", 0)
    keepdims = kw.get("keepdims", False)
    dtype = kw.get("dtype")
    if ufunc is np.add:
        if a.dtype == BOOL:
            return wrap(np.add.reduce(a.astype(I32), axis=axis, keepdims=keepdims))
        if a.dtype == BF16 or a.dtype == np.dtype(np.float16):
            # jnp reductions upcast half types, accumulate in f32, cast back
            r = np.add.reduce(a.astype(F32), axis=axis, keepdims=keepdims, dtype=F32)
            return wrap(r.astype(dtype or a.dtype))
        return wrap(np.add.reduce(a, axis=axis, keepdims=keepdims, dtype=dtype))
    if ufunc in (np.maximum, np.minimum, np.logical_and, np.logical_or):
        cdt = _compute_dtype(a.dtype)
        r = ufunc.reduce(a.astype(cdt), axis=axis, keepdims=keepdims)
        return wrap(np.asarray(r).astype(a.dtype))
    raise NotImplementedError(f"jax_shim: reduce of {ufunc}")


# ---------------------------------------------------------------------------
# jax.numpy
# ---------------------------------------------------------------------------
def _mk_jnp():
    m = types.ModuleType("jax.numpy")
    m.bfloat16 = ml_dtypes.bfloat16
    m.float32 = np.float32
    m.float16 = np.float16
    m.int32 = np.int32
    m.int8 = np.int8
    m.uint32 = np.uint32
    m.bool_ = np.bool_
    m.ndarray = JArr
    m.finfo = ml_dtypes.finfo
    m.iinfo = np.iinfo
    m.dtype = np.dtype

    def asarray(x, dtype=None):
        if dtype is None:
            if _is_weak(x):
                dtype = result_dtype(x)
            return wrap(np.asarray(x) if not isinstance(x, np.ndarray) else x)
        return wrap(np.asarray(x).astype(dtype))
    m.asarray = m.array = asarray

    def arange(*args, dtype=None):
        r = np.arange(*args)
        if dtype is None:
            dtype = I32 if r.dtype.kind in "iu" else F32
        return wrap(r.astype(dtype))
    m.arange = arange
    m.zeros = lambda shape, dtype=F32: wrap(np.zeros(shape, dtype))
    m.ones = lambda shape, dtype=F32: wrap(np.ones(shape, dtype))
    m.full = lambda shape, v, dtype=None: wrap(np.full(shape, v, dtype or result_dtype(v)))
    m.zeros_like = lambda x, dtype=None: wrap(np.zeros(np.shape(x), dtype or np.asarray(x).dtype))

    def _unary(f):
        def g(x):
            if _is_weak(x):                # weak f32 result stays a Python scalar
                return float(f(np.asarray(x, F32)))
            return f(wrap(x) if not isinstance(x, JArr) else x)
        return g
    for name in ("exp", "exp2", "log", "sqrt", "cos", "sin", "tanh", "abs", "negative",
                 "floor", "ceil", "square"):
        setattr(m, name, _unary(getattr(np, name)))
    m.rsqrt = lambda x: 1.0 / m.sqrt(x)
    m.maximum = lambda a, b: np.maximum(_as_j(a), b)
    m.minimum = lambda a, b: np.minimum(_as_j(a), b)
    m.logical_and = lambda a, b: np.logical_and(_as_j(a), b)

    def where(c, x, y):
        dt = result_dtype(x, y)
        xv = np.asarray(x).astype(dt)
        yv = np.asarray(y).astype(dt)
        return wrap(np.where(np.asarray(c), xv, yv))
    m.where = where

    def einsum(eq, *ops, preferred_element_type=None, precision=None, optimize=None):
        dt = result_dtype(*ops)
        cdt = _compute_dtype(dt)
        arrs = [np.asarray(_plain(o)).astype(cdt) for o in ops]
        r = np.einsum(eq, *arrs, optimize=True)
        return wrap(np.asarray(r, cdt).astype(preferred_element_type or dt))
    m.einsum = einsum
    m.dot = lambda a, b, preferred_element_type=None: einsum(
        "...i,i...->...", a, b, preferred_element_type=preferred_element_type) \
        if np.ndim(b) == 1 else _matmul(a, b, preferred_element_type)
    m.matmul = lambda a, b: _matmul(a, b, None)

    m.transpose = lambda x, axes=None: wrap(np.transpose(np.asarray(x), axes))
    m.swapaxes = lambda x, a, b: wrap(np.swapaxes(np.asarray(x), a, b))
    m.reshape = lambda x, shape: wrap(np.reshape(np.asarray(x), shape))
    m.repeat = lambda x, r, axis=None: wrap(np.repeat(np.asarray(x), r, axis=axis))
    m.take = lambda x, idx, axis=None: wrap(np.take(np.asarray(x), np.asarray(idx), axis=axis))
    m.broadcast_to = lambda x, shape: wrap(np.broadcast_to(np.asarray(x), shape))
    m.expand_dims = lambda x, axis: wrap(np.expand_dims(np.asarray(x), axis))
    m.tril = lambda x, k=0: wrap(np.tril(np.asarray(x), k))

    def stack(xs, axis=0):
        dt = result_dtype(*xs)
        return wrap(np.stack([np.asarray(x).astype(dt) for x in xs], axis=axis))
    m.stack = stack

    def concatenate(xs, axis=0):
        dt = result_dtype(*xs)
        return wrap(np.concatenate([np.asarray(x).astype(dt) for x in xs], axis=axis))
    m.concatenate = concatenate

    def pad(x, pad_width, mode="constant", constant_values=0):
        return wrap(np.pad(np.asarray(x), pad_width, mode=mode, constant_values=constant_values))
    m.pad = pad

    m.sum = lambda x, axis=None, keepdims=False, dtype=None: _as_j(x).sum(
        axis=axis, keepdims=keepdims, dtype=dtype)
    m.max = lambda x, axis=None, keepdims=False: _as_j(x).max(axis=axis, keepdims=keepdims)
    m.min = lambda x, axis=None, keepdims=False: _as_j(x).min(axis=axis, keepdims=keepdims)
    m.mean = lambda x, axis=None, keepdims=False: _mean(x, axis, keepdims)
    m.argmax = lambda x, axis=None: wrap(np.argmax(_f32view(x), axis=axis).astype(I32))
    m.issubdtype = np.issubdtype
    m.floating = np.floating
    m.integer = np.integer
    return m


def _as_j(x):
    return x if isinstance(x, JArr) else wrap(x)


def _f32view(x):
    a = np.asarray(_plain(x))
    return a.astype(F32) if a.dtype == BF16 else a


def _mean(x, axis, keepdims):
    a = np.asarray(_plain(x))
    n = a.size if axis is None else np.prod([a.shape[i] for i in np.atleast_1d(axis)])
    s = np.add.reduce(a.astype(F32), axis=axis, keepdims=keepdims)
    return wrap((s / np.float32(n)).astype(a.dtype if a.dtype.kind == "f" or a.dtype == BF16
                                           else F32))


def _matmul(a, b, preferred):
    dt = result_dtype(a, b)
    cdt = _compute_dtype(dt)
    r = np.matmul(np.asarray(_plain(a)).astype(cdt), np.asarray(_plain(b)).astype(cdt))
    return wrap(np.asarray(r, cdt).astype(preferred or dt))


# ---------------------------------------------------------------------------
# jax.lax, jax.nn, jax core
# ---------------------------------------------------------------------------
def _mk_lax():
    m = types.ModuleType("jax.lax")

    def fori_loop(lo, hi, body, init):
        carry = init
        for i in range(int(lo), int(hi)):
            carry = body(np.int32(i), carry)
        return carry
    m.fori_loop = fori_loop

    def cond(pred, true_fn, false_fn, *operands):
        return true_fn(*operands) if bool(pred) else false_fn(*operands)
    m.cond = cond

    def broadcast_in_dim(x, shape, broadcast_dimensions):
        a = np.asarray(x)
        view = [1] * len(shape)
        for src, dst in enumerate(broadcast_dimensions):
            view[dst] = a.shape[src]
        return wrap(np.broadcast_to(a.reshape(view), shape))
    m.broadcast_in_dim = broadcast_in_dim
    m.rsqrt = lambda x: 1.0 / np.sqrt(_as_j(x))
    m.stop_gradient = lambda x: x
    return m


def _mk_nn():
    m = types.ModuleType("jax.nn")

    def softmax(x, axis=-1):
        x = _as_j(x)
        x_max = x.max(axis=axis, keepdims=True)
        unnormalized = np.exp(x - x_max)
        return unnormalized / unnormalized.sum(axis=axis, keepdims=True)
    m.softmax = softmax
    m.silu = lambda x: _as_j(x) * (1.0 / (1.0 + np.exp(-_as_j(x))))
    return m


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape, self.dtype = tuple(int(s) for s in shape), np.dtype(dtype)


def jit(fun=None, **kw):
    if fun is None:
        return lambda f: f
    return fun


def vmap(fun, in_axes=0, out_axes=0):
    def mapped(*args):
        axes = in_axes if isinstance(in_axes, (tuple, list)) else (in_axes,) * len(args)
        n = None
        for a, ax in zip(args, axes):
            if ax is not None and a is not None:
                n = np.shape(a)[ax]
                break
        outs = []
        for i in range(n):
            sub = [a if (ax is None or a is None) else wrap(np.take(np.asarray(a), i, axis=ax))
                   for a, ax in zip(args, axes)]
            outs.append(fun(*sub))
        if isinstance(outs[0], (tuple, list)):
            return type(outs[0])(wrap(np.stack([np.asarray(o[j]) for o in outs], out_axes))
                                 for j in range(len(outs[0])))
        return wrap(np.stack([np.asarray(o) for o in outs], out_axes))
    return mapped


# ---------------------------------------------------------------------------
# Pallas interpreter
# ---------------------------------------------------------------------------
_PID: list[int] = []


class ds:
    def __init__(self, start, size):
        self.start, self.size = start, int(size)


def _norm_index(idx):
    if not isinstance(idx, tuple):
        idx = (idx,)
    out = []
    for c in idx:
        if isinstance(c, ds):
            s = int(c.start)
            out.append(slice(s, s + c.size))
        elif isinstance(c, np.ndarray) and c.ndim == 0:
            out.append(int(c))
        elif isinstance(c, np.ndarray):
            out.append(np.asarray(_plain(c)).astype(np.int64))
        else:
            out.append(c)
    return tuple(out)


class Ref:
    """A kernel's view of one block: reads copy out, writes go through."""

    def __init__(self, view: np.ndarray):
        self.view = view

    shape = property(lambda self: self.view.shape)
    dtype = property(lambda self: self.view.dtype)

    def __getitem__(self, idx):
        if idx is Ellipsis:
            return wrap(self.view.copy())
        return wrap(np.array(self.view[_norm_index(idx)], copy=True))

    def __setitem__(self, idx, value):
        v = np.asarray(_plain(value))
        if idx is Ellipsis:
            self.view[...] = v.astype(self.view.dtype)
        else:
            self.view[_norm_index(idx)] = v.astype(self.view.dtype)


class BlockSpec:
    def __init__(self, block_shape=None, index_map=None, **kw):
        self.block_shape, self.index_map = block_shape, index_map


def _block_view(arr: np.ndarray, spec: BlockSpec, pid) -> np.ndarray:
    if spec.block_shape is None:
        return arr
    bidx = spec.index_map(*[np.int32(p) for p in pid])
    if not isinstance(bidx, tuple):
        bidx = (bidx,)
    sl = []
    for d, (bs, bi) in enumerate(zip(spec.block_shape, bidx)):
        bi = int(bi)
        if bs is None:                    # squeezed dim: element index
            sl.append(min(max(bi, 0), arr.shape[d] - 1))
        else:                             # blocked: block index * block size, clamped
            start = min(max(bi * bs, 0), arr.shape[d] - bs)
            sl.append(slice(start, start + bs))
    return arr[tuple(sl)]


def pallas_call(kernel, *, grid=(), in_specs=None, out_specs=None, out_shape=None, **kw):
    single = not isinstance(out_shape, (list, tuple))
    shapes = [out_shape] if single else list(out_shape)
    ospecs = [out_specs] if single else list(out_specs)

    def call(*args):
        outs = [np.zeros(s.shape, s.dtype) for s in shapes]
        specs = in_specs or [BlockSpec()] * len(args)
        g = grid if isinstance(grid, tuple) else (grid,)
        for pid in itertools.product(*[range(int(n)) for n in g]):
            _PID[:] = list(pid)
            refs = [None if (a is None or sp is None) else Ref(_block_view(np.asarray(_plain(a)),
                                                                          sp, pid))
                    for a, sp in zip(args, specs)]
            orefs = [Ref(_block_view(o, sp, pid)) for o, sp in zip(outs, ospecs)]
            kernel(*refs, *orefs)
        res = [wrap(o) for o in outs]
        return res[0] if single else res
    return call


def program_id(axis):
    return np.int32(_PID[axis])


def cdiv(a, b):
    if isinstance(a, (int, np.integer)) and isinstance(b, (int, np.integer)):
        return (int(a) + int(b) - 1) // int(b)
    return (_as_j(a) + (b - 1)) // b


def pl_dot(a, b, trans_a=False, trans_b=False, allow_tf32=None, precision=None):
    a = np.asarray(_plain(a))
    b = np.asarray(_plain(b))
    if trans_a:
        a = a.T
    if trans_b:
        b = b.T
    out = I32 if np.result_type(a, b).kind in "iu" else F32
    return wrap(np.matmul(a.astype(F32 if out == F32 else I32),
                          b.astype(F32 if out == F32 else I32)).astype(out))


# ---------------------------------------------------------------------------
# installation
# ---------------------------------------------------------------------------
def install() -> types.ModuleType:
    """Register the shim as `jax` (and submodules) in sys.modules."""
    jax = types.ModuleType("jax")
    jnp = _mk_jnp()
    lax = _mk_lax()
    nn = _mk_nn()
    jax.numpy, jax.lax, jax.nn = jnp, lax, nn
    jax.Array = JArr
    jax.jit, jax.vmap = jit, vmap
    jax.ShapeDtypeStruct = ShapeDtypeStruct
    jax.devices = lambda *a: ["cpu"]
    jax.device_put = lambda x, device=None: x
    jax.random = types.SimpleNamespace(PRNGKey=lambda s: s)
    pl = types.ModuleType("jax.experimental.pallas")
    pl.pallas_call, pl.BlockSpec, pl.ds = pallas_call, BlockSpec, ds
    pl.program_id, pl.cdiv, pl.dot = program_id, cdiv, pl_dot
    plgpu = types.ModuleType("jax.experimental.pallas.triton")
    plgpu.CompilerParams = lambda **kw: kw
    pl.triton = plgpu
    exp = types.ModuleType("jax.experimental")
    exp.pallas = pl
    exp.mesh_utils = types.SimpleNamespace(create_device_mesh=lambda *a, **k: None)
    sharding = types.ModuleType("jax.sharding")
    sharding.Mesh = lambda *a, **k: None
    sharding.set_mesh = lambda *a, **k: None
    jax.experimental, jax.sharding = exp, sharding
    for name, mod in {"jax": jax, "jax.numpy": jnp, "jax.lax": lax, "jax.nn": nn,
                      "jax.experimental": exp, "jax.experimental.pallas": pl,
                      "jax.experimental.pallas.triton": plgpu,
                      "jax.experimental.mesh_utils": exp.mesh_utils,
                      "jax.sharding": sharding}.items():
        sys.modules[name] = mod
    return jax


def bf16_array(x) -> JArr:
    return wrap(np.asarray(x).astype(BF16))


__all__ = ["install", "JArr", "wrap", "bf16_array", "BF16", "F32", "I32", "result_dtype",
           "math"]
