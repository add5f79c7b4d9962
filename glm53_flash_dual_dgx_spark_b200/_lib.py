"""ctypes binding of ``libnvfp4kv.so`` (the C ABI declared in ``include/nvfp4kv.h``).

This is the whole host/device boundary: plain pointers, sizes and a stream handle.  The
library must be built (``python -m glm53_flash_dual_dgx_spark_b200.build``); there is no
CPU or Python fallback, so a missing library raises at first use.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("NVFP4KV_LIB", os.path.join(HERE, "libnvfp4kv.so"))

# Return and device-error codes (include/nvfp4kv.h).
OK, EINVAL, EWORKSPACE, ECUDA = 0, 1, 2, 3
DEVERR_TIMEOUT, DEVERR_BAD_SLOT, DEVERR_BAD_INDEX, DEVERR_BAD_PAGE, DEVERR_SEQ_LEN = 1, 2, 4, 8, 16
DEVERR_CAPACITY = 32
DTYPE_BF16, DTYPE_F16 = 0, 1
DIV_IEEE, DIV_TRITON = 0, 1
INDEX_I64, INDEX_I32 = 0, 1

# Every symbol include/nvfp4kv.h declares, with its ctypes signature.
_P, _I, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "nvfp4kv_version": (_I, []),
    "nvfp4kv_last_error": (ctypes.c_char_p, []),
    "nvfp4kv_append": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, _I, _P, _P]),
    "nvfp4kv_gather_ds656": (_I, [_P, _I64, _P, _I64, _P, _P]),
    "nvfp4kv_set_gather_division": (_I, [_I]),
    "nvfp4kv_get_gather_division": (_I, []),
    "nvfp4kv_dequant_bf16": (_I, [_P, _I64, _P, _I, _I64, _P, _P, _P]),
    "nvfp4kv_dedup_gather_ds656": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I64, _P, _P, _P]),
    "nvfp4kv_dedup_workspace_ints": (_I, [_I64, _I64, ctypes.POINTER(_I64)]),
    "nvfp4kv_mla_decode": (_I, [_P, _I64, _I64, _I64,          # q + strides
                                _P, _I64,                      # pool, pool_rows
                                _P, _I64,                      # tables, tables_stride
                                _P,                            # seq_lens
                                _I, _I, _I, _I, _I,            # batch, q_len, heads, dim_qk, rank
                                _I, _I, _I,                    # topk, page_size, max_seq_len
                                _F, _F,                        # bmm1, bmm2
                                _P, _I64, _I64, _I64,          # out + strides
                                _P, _SZ,                       # workspace
                                _P, _P]),                      # err_flag, stream
    "nvfp4kv_mla_decode_lse": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P,
                                    _I, _I, _I, _I, _I, _I, _I, _I, _F, _F,
                                    _P, _I64, _I64, _I64,
                                    _P,                         # lse
                                    _P, _SZ, _P, _P]),          # workspace, err_flag, stream
    "nvfp4kv_mla_decode_workspace_size": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "nvfp4kv_mla_decode_plan": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "nvfp4kv_set_kernel_events": (_I, [_P, _P]),
    "nvfp4kv_selftest_bounded_wait": (_I, [_P, _P]),
    "nvfp4kv_append_rope": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _P, _P]),
    "nvfp4kv_gather_ds656_rope": (_I, [_P, _P, _I64, _P, _I64, _P, _P]),
    "nvfp4kv_mla_decode_rope": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P,   # q + strides, pool, rows, rope
                                     _P, _I64, _P,
                                     _I, _I, _I, _I, _I, _I, _I, _I, _F, _F,
                                     _P, _I64, _I64, _I64,
                                     _P, _SZ, _P, _P]),
    "nvfp4kv_mla_decode_rope_workspace_size": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "nvfp4kv_index_append": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _P, _P]),
    "nvfp4kv_index_topk": (_I, [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _P,
                                _I, _I, _I, _I, _I, _P, _P, _P, _SZ, _P, _P]),
    "nvfp4kv_index_topk_workspace_size": (_I, [_I, _I, ctypes.POINTER(_SZ)]),
    "nvfp4kv_mla_decode_static": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P,
                                       _I, _I, _I, _I, _I, _I, _I, _I, _F, _F,
                                       _P, _I64, _I64, _I64,
                                       _P, _P]),                # err_flag, stream
}


class Nvfp4kvError(RuntimeError):
    """A C-ABI call returned a non-OK code."""


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python -m glm53_flash_dual_dgx_spark_b200.build` (no CPU fallback exists)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().nvfp4kv_last_error()
        raise Nvfp4kvError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")
