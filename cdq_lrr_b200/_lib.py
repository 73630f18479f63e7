"""ctypes binding of libcdq_b200.so (the C ABI declared in include/cdq.h).

The library is built in-tree by ``cdq_lrr_b200.build`` and loaded from the
package directory. There is no fallback: if the library is missing or does
not load, every product entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcdq_b200.so"

STATUS = {
    0: "CDQ_OK", 1: "CDQ_ERR_SHAPE", 2: "CDQ_ERR_STATES", 3: "CDQ_ERR_ARG", 4: "CDQ_ERR_CUDA",
    5: "CDQ_ERR_FORMAT", 6: "CDQ_ERR_CAPACITY", 7: "CDQ_ERR_WORKSPACE", 8: "CDQ_ERR_UNSUPPORTED",
}
MAX_BATCH = 64
MAX_COLS = 65536
MAX_JOBS = 192  # jobs per grouped launch (the launch record fits the kernel-parameter space)
QUANT_NO_TOPK_GUARD = 1  # CDQ_QUANT_NO_TOPK_GUARD


class CdqError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {STATUS.get(status, status)}")


class cdq_packed(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("n_states", C.c_int32),
                ("reserved0", C.c_int32), ("n_res", C.c_int64),
                ("units", C.c_void_p), ("res_ptr", C.c_void_p),
                ("res_ent", C.c_void_p), ("res_q", C.c_void_p)]


class cdq_sizes(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "row_blocks", "tile_pairs", "res_groups", "units_bytes", "res_ptr_count",
        "max_res", "linear_workspace_bytes", "quantize_workspace_bytes")]


class cdq_ipc_handle(C.Structure):
    _fields_ = [("bytes", C.c_uint8 * 64)]


AR_MAX_RANKS = 8  # CDQ_AR_MAX_RANKS


class cdq_gemv_job(C.Structure):
    _fields_ = [("w", cdq_packed), ("x", C.c_void_p), ("y", C.c_void_p), ("bias", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_int64),
                ("out_f32", C.c_int32), ("reserved0", C.c_int32)]


class cdq_step_layer(C.Structure):
    _fields_ = [("q", cdq_gemv_job), ("k", cdq_gemv_job), ("v", cdq_gemv_job), ("o", cdq_gemv_job),
                ("gate", cdq_gemv_job), ("up", cdq_gemv_job), ("down", cdq_gemv_job),
                ("ln1", C.c_void_p), ("ln2", C.c_void_p), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p)]


class cdq_step_model(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("heads", C.c_int32), ("kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("inter", C.c_int32), ("max_len", C.c_int32), ("token_cap", C.c_int32),
                ("vocab", C.c_int64), ("eps", C.c_float), ("scale", C.c_float)] + [
                (n, C.c_void_p) for n in ("embed", "norm_w", "lm_w", "cos_t", "sin_t", "pos", "ids", "tokens",
                                          "count", "best", "next", "logits", "h0", "h1", "q", "k", "v", "att",
                                          "o", "g", "u", "dn")]


class cdq_quant_info(C.Structure):
    _fields_ = [("n_res", C.c_int64), ("k", C.c_int64), ("threshold", C.c_float),
                ("topk_fallback", C.c_int32), ("mask_count", C.c_int64)]


class cdq_file_tensor(C.Structure):
    _fields_ = [("name", C.c_char * 256), ("rows", C.c_int32), ("cols", C.c_int32),
                ("n_tiles", C.c_int64), ("n_res", C.c_int64), ("record_offset", C.c_int64),
                ("record_bytes", C.c_int64)]


_P = C.c_void_p
_SIGS = {
    "cdq_get_sizes": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_double, C.c_int32,
                                C.POINTER(cdq_sizes)]),
    "cdq_version": (C.c_char_p, []),
    "cdq_linear": (C.c_int, [C.POINTER(cdq_packed), _P, C.c_int64, _P, _P, _P, C.c_size_t, _P]),
    "cdq_linear_f32": (C.c_int, [C.POINTER(cdq_packed), _P, C.c_int64, _P, _P, _P, C.c_size_t, _P]),
    "cdq_linear_noalloc": (C.c_int, [C.POINTER(cdq_packed), _P, C.c_int64, _P, _P, _P]),
    "cdq_linear_grouped": (C.c_int, [C.POINTER(cdq_gemv_job), C.c_int32, C.c_int64, _P]),
    "cdq_set_tile_min_batch": (C.c_int, [C.c_int32]),
    "cdq_ar_create": (C.c_int, [C.c_int64, C.POINTER(C.c_void_p), C.POINTER(cdq_ipc_handle)]),
    "cdq_ar_open": (C.c_int, [C.POINTER(cdq_ipc_handle), C.POINTER(C.c_void_p)]),
    "cdq_ar_close": (C.c_int, [C.c_void_p]),
    "cdq_ar_destroy": (C.c_int, [C.c_void_p]),
    "cdq_allreduce_f32": (C.c_int, [C.POINTER(C.c_void_p), C.c_int32, C.c_int32, C.c_int64, C.c_void_p,
                                    C.c_int64, C.c_void_p]),
    "cdq_ar_error": (C.c_int, [C.POINTER(C.c_int32)]),
    "cdq_ar_clear_error": (C.c_int, []),
    "cdq_ar_set_spin_limit": (C.c_int, [C.c_int64]),
    "cdq_pack_from_reference_device": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P, C.c_int64,
                                                 C.POINTER(cdq_packed), _P, _P]),
    "cdq_check_device_pack": (C.c_int, [C.POINTER(cdq_packed), _P, _P]),
    "cdq_step_table_bytes": (C.c_int, [C.c_int32, C.POINTER(C.c_int64)]),
    "cdq_step_prepare": (C.c_int, [C.POINTER(cdq_step_model), C.POINTER(cdq_step_layer), _P]),
    "cdq_decode_step": (C.c_int, [_P, C.c_int32, _P]),
    "cdq_step_error": (C.c_int, [_P, C.POINTER(C.c_int32)]),
    "cdq_step_reset": (C.c_int, [_P, _P]),
    "cdq_file_checkpoints": (C.c_int, [_P, C.c_int64, C.c_int32, C.POINTER(cdq_file_tensor), C.c_int32, _P, _P]),
    "cdq_file_decode_device": (C.c_int, [_P, C.c_int64, C.c_int32, C.c_int64, C.c_int64, C.c_int32, _P, _P,
                                         _P, _P, _P, _P, _P, _P]),
    "cdq_compare_stats": (C.c_int, [_P, _P, C.c_int64, C.c_int32, _P, _P, C.c_int64, _P]),
    "cdq_add_rmsnorm": (C.c_int, [_P, _P, _P, C.c_float, _P, C.c_int32, _P]),
    "cdq_attn_decode": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                  C.c_float, _P, _P]),
    "cdq_silu_mul": (C.c_int, [_P, _P, _P, C.c_int64, _P]),
    "cdq_decode_advance": (C.c_int, [_P, _P, _P, _P, _P, C.c_int32, _P]),
    "cdq_embed_rmsnorm": (C.c_int, [_P, _P, C.c_int64, _P, _P, C.c_float, _P, C.c_int32, _P]),
    "cdq_lm_head_argmax": (C.c_int, [_P, _P, C.c_int32, C.c_int32, _P, _P, _P, _P]),
    "cdq_add_rmsnorm_rows": (C.c_int, [_P, _P, _P, C.c_float, _P, C.c_int32, C.c_int32, _P]),
    "cdq_embed_rmsnorm_rows": (C.c_int, [_P, _P, C.c_int64, _P, _P, C.c_float, _P, C.c_int32, C.c_int32, _P]),
    "cdq_lm_head_argmax_rows": (C.c_int, [_P, _P, C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P]),
    "cdq_attn_decode_multi": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32,
                                        C.c_int32, C.c_float, _P, C.c_int32, _P]),
    "cdq_kernel_error": (C.c_int, [C.POINTER(C.c_int32)]),
    "cdq_dequant": (C.c_int, [C.POINTER(cdq_packed), _P, _P]),
    "cdq_quantize": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.c_double,
                               C.POINTER(cdq_packed), _P, _P, C.c_size_t, _P]),
    "cdq_quantize_ex": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.c_double, C.c_int32, C.c_int64,
                                  C.POINTER(cdq_packed), _P, _P, C.c_size_t, _P]),
    "cdq_pack_tile_indices": (C.c_int, [_P, C.c_int64, C.c_int32, _P]),
    "cdq_unpack_tile_indices": (C.c_int, [_P, C.c_int64, C.c_int32, _P]),
    "cdq_pack_residual_stream": (C.c_int, [_P, _P, C.c_int64, _P]),
    "cdq_unpack_residual_stream": (C.c_int, [_P, C.c_int64, _P, _P]),
    "cdq_host_from_reference": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P,
                                          C.c_int64, C.POINTER(cdq_packed)]),
    "cdq_host_to_reference": (C.c_int, [C.POINTER(cdq_packed), _P, _P, _P, _P]),
    "cdq_file_scan": (C.c_int, [_P, C.c_int64, C.POINTER(C.c_int32), C.POINTER(cdq_file_tensor),
                                C.c_int32, C.POINTER(C.c_int32)]),
    "cdq_file_decode": (C.c_int, [_P, C.c_int64, C.c_int32, C.POINTER(cdq_file_tensor), _P, _P,
                                  _P, _P]),
    "cdq_file_encode_header": (C.c_int, [C.c_int32, C.c_int32, _P, C.c_int64,
                                         C.POINTER(C.c_int64)]),
    "cdq_file_encode_tensor": (C.c_int, [C.c_char_p, C.c_int32, C.c_int32, C.c_int32, _P, _P, _P,
                                         _P, C.c_int64, _P, C.c_int64, C.POINTER(C.c_int64)]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m cdq_lrr_b200.build`")
        h = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, what: str) -> None:
    if status != 0:
        raise CdqError(status, what)


def set_tile_min_batch(m: int) -> None:
    """Batches of at least m rows take the tcgen05 tile path (default 16)."""
    check(lib().cdq_set_tile_min_batch(m), "cdq_set_tile_min_batch")


def ar_error() -> int:
    """The sticky error code of the one-shot all-reduce (0: none)."""
    v = C.c_int32(0)
    check(lib().cdq_ar_error(C.byref(v)), "cdq_ar_error")
    return v.value


def kernel_error() -> int:
    """The sticky in-kernel error code of the fused linear (0: none)."""
    v = C.c_int32(0)
    check(lib().cdq_kernel_error(C.byref(v)), "cdq_kernel_error")
    return v.value


def sizes(rows: int, cols: int, n_states: int, stc_frac: float = 0.0156,
          max_batch: int = MAX_BATCH) -> cdq_sizes:
    s = cdq_sizes()
    check(lib().cdq_get_sizes(rows, cols, n_states, stc_frac, max_batch, C.byref(s)), "cdq_get_sizes")
    return s
