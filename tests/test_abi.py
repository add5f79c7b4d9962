"""CPU: the C-ABI library loads, exports every symbol include/nvfp4kv.h declares, and its
argument checks reject bad calls before any kernel launch (no GPU needed for these)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from glm53_flash_dual_dgx_spark_b200 import _lib

HEADER = os.path.join(ROOT, "include", "nvfp4kv.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nvfp4kv_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) == 23, names
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES)


def test_gather_division_mode_switch_without_launch():
    lib = _lib.lib()
    assert lib.nvfp4kv_get_gather_division() == _lib.DIV_IEEE          # the default
    assert lib.nvfp4kv_set_gather_division(7) == _lib.EINVAL
    assert b"NVFP4KV_DIV" in lib.nvfp4kv_last_error()
    try:
        assert lib.nvfp4kv_set_gather_division(_lib.DIV_TRITON) == _lib.OK
        assert lib.nvfp4kv_get_gather_division() == _lib.DIV_TRITON
    finally:
        assert lib.nvfp4kv_set_gather_division(_lib.DIV_IEEE) == _lib.OK


def test_version_and_empty_error():
    lib = _lib.lib()
    assert lib.nvfp4kv_version() >= 100
    assert isinstance(lib.nvfp4kv_last_error(), bytes)


def test_append_argument_checks_without_launch():
    lib = _lib.lib()
    assert lib.nvfp4kv_append(None, 0, 0, 512, None, 0, None, 0, None, None) == _lib.OK  # T == 0
    assert lib.nvfp4kv_append(None, 0, -1, 512, None, 0, None, 0, None, None) == _lib.EINVAL
    assert lib.nvfp4kv_append(None, 0, 4, 512, None, 16, None, 0, None, None) == _lib.EINVAL
    assert b"null" in lib.nvfp4kv_last_error()
    # 8-byte aligned fake pointers never reach a launch: the stride check fails first
    assert lib.nvfp4kv_append(16, 0, 4, 100, 4096, 16, 64, 0, None, None) == _lib.EINVAL
    assert b"src_stride" in lib.nvfp4kv_last_error()
    assert lib.nvfp4kv_append(16, 7, 4, 512, 4096, 16, 64, 0, None, None) == _lib.EINVAL
    assert lib.nvfp4kv_append(16, 0, 4, 512, 4097, 16, 64, 0, None, None) == _lib.EINVAL  # unaligned pool


def test_gather_and_decode_argument_checks_without_launch():
    lib = _lib.lib()
    assert lib.nvfp4kv_gather_ds656(None, 1, None, 0, None, None) == _lib.OK
    assert lib.nvfp4kv_gather_ds656(None, 1, None, 5, None, None) == _lib.EINVAL
    assert lib.nvfp4kv_gather_ds656(4096, 1, 64, 5, 4100, None) == _lib.EINVAL      # unaligned out
    args = dict(q=4096, sb=64 * 576, sq=64 * 576, sh=576, pool=4096, rows=1024, tables=64, ts=16,
                sl=64, B=2, QL=1, H=64, D=576, R=512, topk=0, page=64, msl=1024, s1=1.0, s2=1.0,
                out=4096, ob=64 * 512, oq=64 * 512, oh=512, ws=None, wsb=0, err=None, st=None)

    def call(**kw):
        a = dict(args, **kw)
        return lib.nvfp4kv_mla_decode(a["q"], a["sb"], a["sq"], a["sh"], a["pool"], a["rows"],
                                      a["tables"], a["ts"], a["sl"], a["B"], a["QL"], a["H"], a["D"],
                                      a["R"], a["topk"], a["page"], a["msl"], a["s1"], a["s2"],
                                      a["out"], a["ob"], a["oq"], a["oh"], a["ws"], a["wsb"],
                                      a["err"], a["st"])

    assert call(B=0) == _lib.OK
    assert call(R=256) == _lib.EINVAL
    assert call(D=500) == _lib.EINVAL
    assert call(topk=2048, QL=3) == _lib.EINVAL
    assert call(page=48) == _lib.EINVAL
    assert call(rows=1000) == _lib.EINVAL          # not a multiple of the page size
    assert call(sh=577) == _lib.EINVAL             # q stride not a multiple of 8
    assert call(ws=None, wsb=0) == _lib.EWORKSPACE  # 2 sequences x 1024 tokens need splits
    assert b"workspace" in lib.nvfp4kv_last_error()


def test_static_decode_rejects_oversized_shapes_without_launch():
    """nvfp4kv_mla_decode_static: argument errors come first, then the 32 MiB capacity.  At 64
    heads and q_len 1 the prepared Q (72.25 KB per 64-row query group) exceeds the scratch
    from 454 groups on; neither path reaches a device call."""
    lib = _lib.lib()
    cap = 33554432
    qimg = 65536 + 8192 + 256
    size = ctypes.c_size_t()
    assert lib.nvfp4kv_mla_decode_workspace_size(453, 1, 64, 8192, 0, ctypes.byref(size)) == _lib.OK
    assert size.value == 453 * qimg <= cap
    assert lib.nvfp4kv_mla_decode_workspace_size(454, 1, 64, 8192, 0, ctypes.byref(size)) == _lib.OK
    assert size.value == 454 * qimg > cap

    def call(B, q=4096, pool=4096, R=512):
        # (q, strides, pool, rows, tables, tstride, seq_lens, B, q_len, H, D, R, topk, page, max_seq,
        #  s1, s2, out, out strides, err, stream): 16-byte aligned fake pointers, never dereferenced
        return lib.nvfp4kv_mla_decode_static(q, 64 * 576, 64 * 576, 576, pool, 1024, 64, 128, 64,
                                             B, 1, 64, 576, R, 0, 64, 8192, 1.0, 1.0,
                                             4096, 64 * 512, 64 * 512, 512, None, None)

    assert call(0) == _lib.OK
    assert call(454) == _lib.EWORKSPACE
    assert b"static scratch" in lib.nvfp4kv_last_error()
    assert call(454, q=None) == _lib.EINVAL           # a null pointer is reported, not the capacity
    assert call(454, pool=4100) == _lib.EINVAL        # so is a misaligned pool
    assert call(454, R=256) == _lib.EINVAL


def test_rope_entry_points_check_arguments_without_launch():
    lib = _lib.lib()
    # append_rope: (k_pe, T, stride, rope_pool, rows, slots, slot dtype, err, stream)
    assert lib.nvfp4kv_append_rope(None, 0, 64, None, 0, None, 0, None, None) == _lib.OK     # T == 0
    assert lib.nvfp4kv_append_rope(4096, 4, 64, None, 16, 64, 0, None, None) == _lib.EINVAL  # null pool
    assert lib.nvfp4kv_append_rope(4096, 4, 32, 4096, 16, 64, 0, None, None) == _lib.EINVAL  # stride < 64
    assert lib.nvfp4kv_append_rope(4096, 4, 64, 4104, 16, 64, 0, None, None) == _lib.EINVAL  # unaligned pool
    assert lib.nvfp4kv_gather_ds656_rope(4096, None, 16, 64, 4, 4096, None) == _lib.EINVAL     # null rope
    assert lib.nvfp4kv_gather_ds656_rope(4096, 4104, 16, 64, 4, 4096, None) == _lib.EINVAL     # unaligned

    def dec(rope=4096, D=576, ws=None, wsb=0):
        return lib.nvfp4kv_mla_decode_rope(4096, 64 * 576, 64 * 576, 576, 4096, 1024, rope, 64, 16, 64,
                                           2, 1, 64, D, 512, 0, 64, 1024, 1.0, 1.0,
                                           4096, 64 * 512, 64 * 512, 512, ws, wsb, None, None)
    assert dec(rope=None) == _lib.EINVAL
    assert dec(D=512) == _lib.EINVAL                     # no rope dims in q
    assert dec() == _lib.EWORKSPACE
    plain, rope = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.nvfp4kv_mla_decode_workspace_size(2, 1, 64, 1024, 0, ctypes.byref(plain)) == _lib.OK
    assert lib.nvfp4kv_mla_decode_rope_workspace_size(2, 1, 64, 1024, 0, ctypes.byref(rope)) == _lib.OK
    # + a 64 x 64 fp32 rope image per query group + 64 rows x 1024 positions of fp32 scores
    assert rope.value == plain.value + 2 * 64 * 64 * 4 + 2 * 64 * 1024 * 4


def test_dedup_workspace_and_argument_checks_without_launch():
    lib = _lib.lib()
    ints = ctypes.c_int64()
    # 4096 pool rows: 4097 marks, one block sum per 4096 marks, min(entries, 4097) values
    assert lib.nvfp4kv_dedup_workspace_ints(4096, 19200, ctypes.byref(ints)) == _lib.OK
    assert ints.value == 4097 + 2 + 4097
    assert lib.nvfp4kv_dedup_workspace_ints(4096, 100, ctypes.byref(ints)) == _lib.OK
    assert ints.value == 4097 + 2 + 100
    assert lib.nvfp4kv_dedup_workspace_ints(0, 100, ctypes.byref(ints)) == _lib.EINVAL
    assert lib.nvfp4kv_dedup_workspace_ints(4096, -1, ctypes.byref(ints)) == _lib.EINVAL
    assert lib.nvfp4kv_dedup_workspace_ints(4096, 1, None) == _lib.EINVAL
    call = lib.nvfp4kv_dedup_gather_ds656
    # (pool, rows, entries, n, ws, ws_ints, tables, scratch, scratch_rows, n_unique, err, stream)
    assert call(None, 4096, 64, 10, 64, 8300, 64, 64, 64, 64, None, None) == _lib.EINVAL    # null pool
    assert call(4096, 4096, 64, -1, 64, 8300, 64, 64, 64, 64, None, None) == _lib.EINVAL    # n < 0
    assert call(4096, 4096, 64, 10, 64, 8300, 64, None, 64, 64, None, None) == _lib.EINVAL  # no scratch
    assert call(4096, 4096, 64, 10, 64, 8300, 64, 4100, 64, 64, None, None) == _lib.EINVAL  # unaligned
    assert call(4096, 0, 64, 10, 64, 8300, 64, 64, 64, 64, None, None) == _lib.EINVAL       # empty pool
    assert call(4096, 4096, 64, 10, 64, 100, 64, 64, 64, 64, None, None) == _lib.EWORKSPACE
    assert b"workspace" in lib.nvfp4kv_last_error()


def test_workspace_size_formula():
    lib = _lib.lib()
    out = ctypes.c_size_t()
    qimg = 65536 + 8192 + 256                      # prepared Q of one 64-row query group
    assert lib.nvfp4kv_mla_decode_workspace_size(16, 1, 64, 8192, 0, ctypes.byref(out)) == _lib.OK
    # 16 query groups on (at least) 148 SMs: up to 9 splits, and 8 of 8 tiles give the same
    # longest split as 9 of 7-8; 64 rows x (512 + 2) floats per split
    assert out.value == 8 * 16 * 64 * 514 * 4 + 16 * qimg
    assert lib.nvfp4kv_mla_decode_workspace_size(256, 1, 64, 8192, 0, ctypes.byref(out)) == _lib.OK
    assert out.value == 256 * qimg                 # enough query groups: no split partials
    assert lib.nvfp4kv_mla_decode_workspace_size(16, 1, 64, 0, 2048, ctypes.byref(out)) == _lib.OK
    assert out.value == 8 * 16 * 64 * 514 * 4 + 16 * qimg   # sparse: 8 splits of 2 tiles
    assert lib.nvfp4kv_mla_decode_workspace_size(-1, 1, 64, 8192, 0, ctypes.byref(out)) == _lib.EINVAL


def test_decode_plan():
    lib = _lib.lib()
    splits, launches = ctypes.c_int(), ctypes.c_int()
    assert lib.nvfp4kv_mla_decode_plan(16, 1, 64, 8192, 0, ctypes.byref(splits), ctypes.byref(launches)) == _lib.OK
    assert (splits.value, launches.value) == (8, 3)        # Q preparation + attention + combine
    assert lib.nvfp4kv_mla_decode_plan(256, 1, 64, 8192, 0, ctypes.byref(splits), ctypes.byref(launches)) == _lib.OK
    assert (splits.value, launches.value) == (1, 2)
    assert lib.nvfp4kv_mla_decode_plan(16, 1, 64, 0, 2048, ctypes.byref(splits), ctypes.byref(launches)) == _lib.OK
    assert (splits.value, launches.value) == (8, 3)        # sparse: same three launches
    assert lib.nvfp4kv_mla_decode_plan(1, 0, 64, 8192, 0, ctypes.byref(splits), ctypes.byref(launches)) == _lib.EINVAL
    assert lib.nvfp4kv_set_kernel_events(None, None) == _lib.OK
    assert lib.nvfp4kv_set_kernel_events(ctypes.c_void_p(1), None) == _lib.EINVAL
    assert lib.nvfp4kv_selftest_bounded_wait(None, None) == _lib.EINVAL   # checked before any launch


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def test_index_topk_argument_checks_without_launch():
    """The page-copy contract of the scoring kernel (pages of at least two 72-byte rows, a
    16-byte aligned pool) and the other argument checks fail before any launch."""
    lib = _lib.lib()

    def call(pool=4096, rows=4096, page=64, heads=64, ws=None, wsb=0, batch=2, q=4096):
        # (q, q_sb, q_sh, w, w_sb, pool, pool_rows, tables, t_stride, seq_lens, batch, heads, page,
        #  max_seq_len, topk, out_rows, out_count, ws, ws_bytes, err, stream)
        return lib.nvfp4kv_index_topk(q, 64 * 128, 128, 4096, 64, pool, rows, 4096, 16, 4096, batch, heads, page,
                                      1024, 2048, 4096, 4096, ws, wsb, None, None)
    assert call(batch=0) == _lib.OK
    assert call(q=None) == _lib.EINVAL
    assert call(heads=32) == _lib.EINVAL
    assert call(page=1) == _lib.EINVAL                   # a one-row page is not a 16-byte run
    assert call(page=48) == _lib.EINVAL                  # not a power of two
    assert call(rows=4000) == _lib.EINVAL                # pages do not divide the pool
    assert call(pool=4104) == _lib.EINVAL                # pool not 16-byte aligned
    assert call() == _lib.EWORKSPACE
    need = ctypes.c_size_t()
    assert lib.nvfp4kv_index_topk_workspace_size(2, 1024, ctypes.byref(need)) == _lib.OK
    assert need.value == 2 * 1024 * 4
    assert call(ws=4100, wsb=need.value) == _lib.EINVAL  # workspace not 16-byte aligned
