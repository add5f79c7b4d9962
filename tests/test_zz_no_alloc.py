"""GPU: nvfp4kv_mla_decode_static (split partials in a fixed device array, no workspace
argument) against nvfp4kv_mla_decode with a caller workspace, both called through the C ABI.

Two static calls in a row must each match the workspace entry point within the decode
tolerance (rtol 2e-2, atol 1e-2); they run the same kernels with the same split plan, so
they are expected to agree bit for bit as well.  After a warm-up call, the two calls must
leave the device's free memory unchanged (nothing is allocated).  The file is named to be collected last and
builds all of its inputs itself, so it passes alone in a fresh process or after other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from glm53_flash_dual_dgx_spark_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 1e-2
SM = 1.0 / 24.0


def _inputs(B, H, ctx, num_pages, sparse_topk, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(num_pages * 64, 512, generator=g).to(torch.bfloat16)
    pool = torch.from_numpy(O.quant_new(x)).cuda().view(num_pages, 64, 288)
    q = torch.randn(B, 1, H, 576, generator=g).to(torch.bfloat16).cuda()
    if sparse_topk:
        tables = torch.stack([torch.randperm(num_pages * 64, generator=g)[:sparse_topk]
                              for _ in range(B)]).to(torch.int32).cuda()
        seq_lens = torch.full((B,), sparse_topk, dtype=torch.int32).cuda()
    else:
        width = (ctx + 63) // 64
        tables = torch.stack([torch.randperm(num_pages, generator=g)[:width]
                              for _ in range(B)]).to(torch.int32).cuda()
        seq_lens = torch.tensor([ctx - 37 * b for b in range(B)], dtype=torch.int32).cuda()
    return q, pool, tables, seq_lens


def _common_args(q, pool, tables, seq_lens, B, H, ctx, sparse_topk, out):
    return [ctypes.c_void_p(q.data_ptr()), q.stride(0), q.stride(1), q.stride(2),
            ctypes.c_void_p(pool.data_ptr()), pool.numel() // 288,
            ctypes.c_void_p(tables.data_ptr()), tables.stride(0),
            ctypes.c_void_p(seq_lens.data_ptr()),
            B, 1, H, 576, 512, sparse_topk, 64, ctx, SM, 1.0,
            ctypes.c_void_p(out.data_ptr()), out.stride(0), out.stride(1), out.stride(2)]


@pytest.mark.parametrize("B,H,ctx,num_pages,sparse_topk", [
    (2, 64, 4096, 80, 0),      # 2 units -> many splits: the partials are in use
    (3, 128, 1000, 20, 0),     # two head groups, ragged lengths
    (4, 64, 2048, 40, 2048),   # sparse top-k rows
])
def test_static_scratch_matches_workspace_entry_point(B, H, ctx, num_pages, sparse_topk):
    lib = _lib.lib()
    torch.cuda.set_device(0)
    q, pool, tables, seq_lens = _inputs(B, H, ctx, num_pages, sparse_topk, seed=B * 7 + H)
    size = ctypes.c_size_t(0)
    _lib.check(lib.nvfp4kv_mla_decode_workspace_size(B, 1, H, ctx, sparse_topk, ctypes.byref(size)),
               "workspace_size")
    assert size.value <= 33554432
    ws = torch.empty(max(size.value, 256), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    ref = torch.empty(B, 1, H, 512, dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.nvfp4kv_mla_decode(*_common_args(q, pool, tables, seq_lens, B, H, ctx, sparse_topk, ref),
                                      ctypes.c_void_p(ws.data_ptr()), size.value,
                                      ctypes.c_void_p(err.data_ptr()), stream), "mla_decode")
    # warm-up call: the first one on a device looks up the scratch array (and, with lazy module
    # loading, may load the module that holds it); every call after it must allocate nothing
    warm = torch.empty(B, 1, H, 512, dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.nvfp4kv_mla_decode_static(*_common_args(q, pool, tables, seq_lens, B, H, ctx, sparse_topk, warm),
                                             ctypes.c_void_p(err.data_ptr()), stream), "mla_decode_static")
    outs = [torch.full((B, 1, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for out in outs:
        _lib.check(lib.nvfp4kv_mla_decode_static(*_common_args(q, pool, tables, seq_lens, B, H, ctx,
                                                               sparse_topk, out),
                                                 ctypes.c_void_p(err.data_ptr()), stream),
                   "mla_decode_static")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "a static call changed the device's free memory"
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    r = ref.float().cpu().numpy()
    assert np.isfinite(r).all()
    for k, out in enumerate(outs):
        o = out.float().cpu().numpy()
        assert np.isfinite(o).all(), f"call {k}: non-finite output"
        assert np.allclose(o, r, rtol=RTOL, atol=ATOL), f"call {k}: max |diff| {np.abs(o - r).max()}"
        assert np.array_equal(o, r), f"call {k}: not bit-identical to the workspace entry point"
