"""GPU: build_scratch_sync_free (nvfp4kv_dedup_gather_ds656) against the reference's large-step
branch of build_scratch (runtime:177-182, torch.unique + _gather), as the oracle restates it.

tables must be identical, and the first ceil(n_unique / 64) pages of the scratch byte-identical
(gathered rows, then zeros to the end of the last page); the call must not synchronise with the
host, and it must replay from a CUDA graph.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def _pool(rows, seed):
    g = torch.Generator().manual_seed(seed)
    pool_np = O.quant_new(torch.randn(rows, 512, generator=g).to(torch.bfloat16))
    return pool_np, torch.from_numpy(pool_np).cuda().view(rows // 64, 64, 288)


def _tables(T, K, rows, seed, pad=0.1, distinct=None):
    g = np.random.default_rng(seed)
    src = np.arange(rows) if distinct is None else g.choice(rows, distinct, replace=False)
    bt = g.choice(src, size=(T, 1, K)).astype(np.int32)
    bt[g.random(bt.shape) < pad] = -1
    return bt


def _check(rt, pool_np, pool, bt):
    scratch, tables, nu = rt.build_scratch_sync_free(pool, torch.from_numpy(bt).cuda())
    ref_scratch, ref_tables = O.build_scratch(pool_np, bt)
    assert int(nu.item()) == len(np.unique(bt))
    assert np.array_equal(tables.cpu().numpy(), ref_tables)
    P = ref_scratch.shape[0]
    got = scratch[:P].cpu().numpy()
    bad = np.argwhere(got != ref_scratch)
    assert bad.size == 0, f"{len(bad)} bytes differ, first {bad[:4].tolist()}"


@pytest.mark.parametrize("T,K,distinct,pad", [(300, 64, None, 0.1), (256, 2048, 3000, 0.02),
                                              (193, 16, 50, 0.0), (400, 128, None, 0.5)])
def test_dedup_matches_reference_branch(rt, T, K, distinct, pad):
    pool_np, pool = _pool(8192, seed=T)
    _check(rt, pool_np, pool, _tables(T, K, 8192, seed=K, pad=pad, distinct=distinct))
    assert rt.device_errors() == 0


def test_dedup_all_padding_and_single_row(rt):
    pool_np, pool = _pool(256, seed=3)
    _check(rt, pool_np, pool, np.full((200, 1, 8), -1, np.int32))      # only -1: one row (row 0)
    _check(rt, pool_np, pool, np.full((200, 1, 8), 255, np.int32))     # one distinct row, the last
    assert rt.device_errors() == 0


def test_dedup_is_sync_free_and_graph_capturable(rt):
    pool_np, pool = _pool(4096, seed=5)
    bt0 = torch.from_numpy(_tables(256, 64, 4096, seed=1)).cuda()
    rt.build_scratch_sync_free(pool, bt0)                # warm-up: workspace allocated once
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")              # any host synchronisation raises
    try:
        rt.build_scratch_sync_free(pool, bt0)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    bt = bt0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            scratch, tables, nu = rt.build_scratch_sync_free(pool, bt)
    torch.cuda.current_stream().wait_stream(s)
    for seed in (7, 8):
        new = _tables(256, 64, 4096, seed=seed, distinct=700)
        bt.copy_(torch.from_numpy(new))
        graph.replay()
        torch.cuda.synchronize()
        ref_scratch, ref_tables = O.build_scratch(pool_np, new)
        assert int(nu.item()) == len(np.unique(new))
        assert np.array_equal(tables.cpu().numpy(), ref_tables)
        P = ref_scratch.shape[0]
        assert np.array_equal(scratch[:P].cpu().numpy(), ref_scratch)
    del graph
    assert rt.device_errors() == 0


def test_dedup_flags_bad_entries_and_capacity(rt):
    pool_np, pool = _pool(1024, seed=9)
    bt = _tables(200, 8, 1024, seed=2)
    bt[0, 0, 0] = 5000                                   # beyond the pool
    bt[1, 0, 1] = -7
    rt.build_scratch_sync_free(pool, torch.from_numpy(bt).cuda())
    assert rt.device_errors() & 4                        # NVFP4KV_DEVERR_BAD_INDEX
    bt = _tables(200, 8, 1024, seed=3, pad=0.0)
    scratch, tables, nu = rt.build_scratch_sync_free(pool, torch.from_numpy(bt).cuda(), capacity_rows=100)
    assert int(nu.item()) == len(np.unique(bt)) > 100
    assert rt.device_errors() & 32                       # NVFP4KV_DEVERR_CAPACITY
    ref_scratch, ref_tables = O.build_scratch(pool_np, bt)
    assert np.array_equal(tables.cpu().numpy(), ref_tables)
    assert np.array_equal(scratch.view(-1, 656)[:100].cpu().numpy(), ref_scratch.reshape(-1, 656)[:100])


def test_build_scratch_large_step_uses_the_device_dedup(rt, monkeypatch):
    """build_scratch's large-step branch is the device dedup by default (GLM53_NVFP4_UNIQUE=1
    selects torch.unique): same tables as the reference branch, its pages first, no host
    sync, and a persistent scratch that later calls reuse instead of allocating."""
    pool_np, pool = _pool(2048, seed=12)
    bt = _tables(256, 32, 2048, seed=4, distinct=500)
    ref_scratch, ref_tables = O.build_scratch(pool_np, bt)
    monkeypatch.setattr(rt, "_UNIQUE", False)
    btd = torch.from_numpy(bt).cuda()
    rt.build_scratch(pool, btd)                          # allocates the workspace once
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        scratch, tables = rt.build_scratch(pool, btd)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    assert np.array_equal(tables.cpu().numpy(), ref_tables)
    P = ref_scratch.shape[0]
    assert np.array_equal(scratch[:P].cpu().numpy(), ref_scratch)
    assert rt.device_errors() == 0
    again, _ = rt.build_scratch(pool, btd)
    assert again.data_ptr() == scratch.data_ptr()        # the persistent buffer, not a new one
    monkeypatch.setattr(rt, "_SYNC_FREE_ROWS", 512)      # a capped scratch: 500 distinct rows fit
    capped, tables = rt.build_scratch(pool, btd)
    assert capped.shape[0] == 8
    assert np.array_equal(tables.cpu().numpy(), ref_tables)
    assert np.array_equal(capped[:P].cpu().numpy(), ref_scratch)
    assert rt.device_errors() == 0
