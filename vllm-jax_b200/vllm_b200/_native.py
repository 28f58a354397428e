"""ctypes binding of libvjattn.so, the sm_100a kernel library.

There is no fallback: if the library is missing or fails to load, every op
raises. The C prototypes mirror include/vjattn.h one to one.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libvjattn.so"
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

c_int, c_i32, c_i64, c_f32, c_sz, c_vp = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p)

# name -> (restype, argtypes); must match include/vjattn.h
PROTOTYPES: dict[str, tuple] = {
    "vj_get_last_error": (ctypes.c_char_p, []),
    "vj_version": (c_int, []),
    "vj_kv_store_qknorm_rope": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,   # q,k,v, qw,kw, positions, slots
        c_vp, c_vp, c_vp, c_vp,                     # q_out, k_out, k_cache, v_cache
        c_i64, c_i32, c_i32, c_i32, c_i64, c_i32,   # T, Hq, Hkv, D, nb, bs
        c_i64, c_i64, c_i64,                        # strides (block, token, head)
        c_i64, c_i64, c_i64,                        # q/k/v row strides (0 = packed)
        c_vp, c_i32,                                # rope_table, rope_table_len
        c_f32, c_f32, c_i32, c_vp]),                # eps, theta, flags, stream
    "vj_rope_table_bytes": (c_sz, [c_i32, c_i32]),
    "vj_kv_store_timeouts": (c_int, [c_vp, c_i32]),
    "vj_rope_table_build": (c_int, [c_vp, c_i32, c_i32, c_f32, c_vp]),
    "vj_paged_decode_workspace_size": (c_sz, [c_i32, c_i32, c_i32, c_i32]),
    "vj_paged_decode": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,         # q, k_cache, v_cache, bt, lens, out
        c_i32, c_i32, c_i32, c_i32, c_i64, c_i32,   # B, Hq, Hkv, D, nb, bs
        c_i32, c_i32,                               # bt_width, bt_stride
        c_i64, c_i64, c_i64,                        # strides
        c_f32, c_i32, c_vp, c_sz, c_vp]),           # scale, max_chunks, ws, ws_bytes, stream
    "vj_paged_decode_planned": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,         # q, k_cache, v_cache, bt, lens, out
        c_i32, c_i32, c_i32, c_i32, c_i64, c_i32,   # B, Hq, Hkv, D, nb, bs
        c_i32, c_i32,                               # bt_width, bt_stride
        c_i64, c_i64, c_i64,                        # strides
        c_f32, c_i32, c_vp, c_sz, c_vp]),           # scale, max_chunks, ws, ws_bytes, stream
    "vj_paged_decode_noalloc_scratch_bytes": (c_sz, []),
    "vj_paged_decode_noalloc": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,         # q, k_cache, v_cache, bt, lens, out
        c_i32, c_i32, c_i32, c_i32, c_i64, c_i32,   # B, Hq, Hkv, D, nb, bs
        c_i32, c_i32,                               # bt_width, bt_stride
        c_i64, c_i64, c_i64,                        # strides
        c_f32, c_vp]),                              # scale, stream
    "vj_paged_prefill": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,   # q, k, v, bt, cu_q, ctx_lens, out
        c_i64, c_i32, c_i32, c_i32, c_i32,          # T, S, Hq, Hkv, D
        c_i64, c_i32, c_i32, c_i32,                 # nb, bs, bt_width, bt_stride
        c_i64, c_i64, c_i64,                        # strides
        c_i32, c_f32, c_vp, c_vp]),                 # max_seqlen_q, scale, err, stream
    "vj_paged_attention_mixed_workspace_size": (c_sz, [c_i32, c_i32, c_i32, c_i32]),
    "vj_paged_attention_mixed": (c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,   # q, k, v, bt, cu_q, ctx_lens, out
        c_i64, c_i32, c_i32, c_i32, c_i32, c_i32,   # T, S, num_decode, Hq, Hkv, D
        c_i64, c_i32, c_i32, c_i32,                 # nb, bs, bt_width, bt_stride
        c_i64, c_i64, c_i64,                        # strides
        c_i32, c_f32, c_i32, c_i32,                 # max_seqlen_q, scale, max_chunks, plan
        c_vp, c_sz, c_vp, c_vp]),                   # ws, ws_bytes, err, stream
    "vj_build_metadata": (c_int, [
        c_i32, c_vp, c_vp, c_vp, c_i32,             # mode, slots, starts, lens, num_seqs
        c_vp, c_i32, c_vp, c_vp, c_i32,             # token_table, stride, block_pool, nblocks, bt_stride
        c_i32, c_i32, c_i32, c_i32, c_i32,          # block_size, width, bucket_tokens, bucket_batch, flags
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,         # ids, positions, slots, block_tables, cu, ctx
        c_vp, c_vp]),                               # error_flag, stream
    "vj_add_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_f32, c_vp]),
    "vj_silu_mul": (c_int, [c_vp, c_vp, c_i64, c_i32, c_vp]),
    "vj_decode_gemm_workspace_size": (c_sz, [c_i64, c_i32, c_i32, c_i32, c_i32]),
    "vj_pack_weight_tiles": (c_int, [c_vp, c_vp, c_i32, c_i32, c_i32, c_vp]),
    "vj_decode_gemm": (c_int, [
        c_vp, c_i64, c_vp, c_i32, c_vp, c_i64,      # x, ldx, w, layout, out, ldo
        c_i64, c_i32, c_i32, c_i32, c_i32,          # rows, n, k, mode, splits
        c_vp, c_sz, c_vp, c_vp]),                   # ws, ws_bytes, err, stream
    "vj_qkv_gemm_kv_store": (c_int, [
        c_vp, c_i64, c_vp, c_i32,                   # x, ldx, w_qkv, layout
        c_vp, c_vp, c_vp, c_vp,                     # qw, kw, positions, slots
        c_vp, c_vp, c_vp,                           # q_out, k_cache, v_cache
        c_i64, c_i32, c_i32, c_i32, c_i32,          # T, hidden, Hq, Hkv, D
        c_i64, c_i32, c_i64, c_i64, c_i64,          # nb, bs, strides (block, token, head)
        c_vp, c_i32, c_f32, c_f32, c_i32, c_i32,    # table, table_len, eps, theta, flags, splits
        c_vp, c_sz, c_vp, c_vp]),                   # ws, ws_bytes, err, stream
    "vj_scatter_rows": (c_int, [c_vp, c_vp, c_i32, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "vj_argmax_append": (c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_i32, c_vp, c_vp,
                                 c_vp]),
    "vj_tp_grid": (c_i32, []),
    "vj_tp_flags_bytes": (c_sz, [c_i32]),
    "vj_comm_alloc": (c_int, [c_sz, c_vp]),
    "vj_comm_free": (c_int, [c_vp]),
    "vj_ipc_get_handle": (c_int, [c_vp, c_vp]),
    "vj_ipc_open_handle": (c_int, [c_vp, c_vp]),
    "vj_ipc_close_handle": (c_int, [c_vp]),
    "vj_allreduce_add_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp,
                                         c_vp, c_i64, c_i32, ctypes.c_float, c_vp]),
    "vj_sample": (c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                          c_i32, c_vp, c_vp, c_vp]),
}

# vj_status codes (include/vjattn.h)
VJ_OK, VJ_ERR_INVALID_ARGUMENT, VJ_ERR_UNSUPPORTED, VJ_ERR_WORKSPACE, VJ_ERR_CUDA = range(5)
VJ_KV_NORM, VJ_KV_ROPE, VJ_KV_WRAP_NEGATIVE = 1, 2, 4
VJ_KV_QSCALE_DIV_SQRT_D, VJ_KV_QSCALE_MUL_RSQRT_D = 8, 16
VJ_META_PREFILL, VJ_META_DECODE, VJ_META_RANGES = 0, 1, 2
VJ_META_LAST_BLOCK_SLOT = 1
VJ_GEMM_PLAIN, VJ_GEMM_SWIGLU = 0, 1
VJ_WEIGHTS_ROW_MAJOR, VJ_WEIGHTS_TILED = 0, 1


class VJError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[vj_status {status}] {msg}")
        self.status = status


def lib_path() -> Path:
    return Path(os.environ.get("VJATTN_LIB", _LIB_PATH))


def load() -> ctypes.CDLL:
    """Load libvjattn.so (once) and bind every prototype; raise if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not path.exists():
                raise RuntimeError(
                    f"{path} not found: build it with `python -m vllm_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(path))
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int) -> None:
    if status != VJ_OK:
        msg = load().vj_get_last_error().decode(errors="replace")
        if status == VJ_ERR_INVALID_ARGUMENT:
            raise ValueError(f"[vj_status {status}] {msg}")
        raise VJError(status, msg)


# kernels launched by one successful call of each entry point
KERNELS_PER_CALL = {"vj_paged_decode": 3, "vj_paged_decode_planned": 2,
                    "vj_paged_decode_noalloc": 3, "vj_paged_prefill": 2,
                    "vj_paged_attention_mixed": 3}
launch_count = 0


def call(name: str, *args) -> None:
    """Call an entry point, raise on a nonzero status, count its kernel launches
    (a CUDA graph replay adds the launches counted while it was captured)."""
    global launch_count
    check(getattr(load(), name)(*args))
    launch_count += KERNELS_PER_CALL.get(name, 1)
