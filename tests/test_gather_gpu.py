"""GPU: the 656-byte gather and build_scratch are byte-identical with the reference, and the
sync-free build_scratch path makes no synchronising call (the properties that
nvfp4-kv/test_syncfree.py pins), plus the bf16 dequantiser against the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def test_gather_matches_reference_golden(rt):
    g = np.load(os.path.join(GOLDEN, "gather_golden.npz"))
    pool = torch.from_numpy(g["pool"]).cuda()
    idx = torch.from_numpy(g["idx"]).cuda()
    out = torch.zeros(idx.shape[0], 656, dtype=torch.uint8, device="cuda")
    rt._gather(pool, idx, out)
    got = out.cpu().numpy()
    bad = np.argwhere(got != g["out_ref"])
    assert bad.size == 0, f"{len(bad)} bytes differ, first {bad[:8].tolist()}"


@pytest.mark.parametrize("T", [3, 5])
def test_build_scratch_matches_reference_golden(rt, T):
    s = np.load(os.path.join(GOLDEN, "scratch_golden.npz"))
    pool = torch.from_numpy(s["pool"]).cuda()
    bt = torch.from_numpy(s[f"bt_{T}"]).cuda()
    rt._bufs.clear()
    sa, ta = rt.build_scratch(pool, bt)
    assert np.array_equal(sa.cpu().numpy(), s[f"sync_scratch_{T}"])
    assert np.array_equal(ta.cpu().numpy(), s[f"sync_tables_{T}"])
    for unique in (True, False):
        sb, tb = _large_step_path(rt, pool, bt, unique)
        ref = s[f"uniq_scratch_{T}"]
        if unique:                                   # the reference's torch.unique branch
            assert np.array_equal(sb.cpu().numpy(), ref)
        else:                                        # device dedup: its pages come first
            assert np.array_equal(sb[:ref.shape[0]].cpu().numpy(), ref)
        assert np.array_equal(tb.cpu().numpy(), s[f"uniq_tables_{T}"])


POOL_ROWS = 100_000


@pytest.fixture(scope="module")
def random_pool():
    torch.manual_seed(0)
    return torch.randint(0, 256, (POOL_ROWS, 288), dtype=torch.uint8, device="cuda")


def _large_step_path(rt, pool, tables, unique):
    """build_scratch's T > _SYNC_FREE_T branch: torch.unique (unique=True, the reference's)
    or the default device dedup."""
    saved = rt._SYNC_FREE_T, rt._UNIQUE
    rt._SYNC_FREE_T, rt._UNIQUE = 0, unique
    try:
        return rt.build_scratch(pool, tables)
    finally:
        rt._SYNC_FREE_T, rt._UNIQUE = saved


@pytest.mark.parametrize("T,K", [(1, 64), (3, 64), (17, 64), (64, 64), (65, 64), (100, 64), (192, 64),
                                 (20, 2048), (65, 2048), (148, 2048), (192, 2048)])
def test_sync_free_equals_unique_path(rt, random_pool, T, K):
    """test_syncfree.py:21-40: byte equality across every table entry, 10% -1 padding,
    cross-token duplicates; and both equal the oracle's gather."""
    idx = torch.randint(0, POOL_ROWS, (T, 1, K), dtype=torch.int32, device="cuda")
    idx[:, :, : K // 4] = idx[:1, :, : K // 4]
    idx[torch.rand(T, 1, K, device="cuda") < 0.1] = -1
    sa, ta = rt.build_scratch(random_pool, idx)
    fa = sa.reshape(-1, 656)[ta.view(-1).long()]
    for unique in (True, False):
        sb, tb = _large_step_path(rt, random_pool, idx, unique)
        fb = sb.reshape(-1, 656)[tb.view(-1).long()]
        assert torch.equal(fa, fb)
    if T * K <= 20000:
        ref = O.gather_ds656(random_pool.cpu().numpy(), idx.view(-1).cpu().numpy())
        assert np.array_equal(fa.cpu().numpy(), ref)


def test_sync_free_path_makes_no_synchronising_call(rt, random_pool):
    """test_syncfree.py:43-51: once the buffers exist, T=148 K=2048 runs with sync debug
    mode set to error."""
    idx = torch.randint(0, POOL_ROWS, (148, 1, 2048), dtype=torch.int32, device="cuda")
    rt.build_scratch(random_pool, idx)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(3):
            rt.build_scratch(random_pool, idx)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()


def test_gather_large_random_rows_vs_oracle(rt, random_pool):
    g = torch.Generator().manual_seed(9)
    idx = torch.randint(-3, POOL_ROWS + 3, (65536,), dtype=torch.int32, generator=g)
    out = torch.empty(65536, 656, dtype=torch.uint8, device="cuda")
    rt._gather(random_pool, idx.cuda(), out)
    ref = O.gather_ds656(random_pool.cpu().numpy(), idx.numpy())
    assert np.array_equal(out.cpu().numpy(), ref)


def test_dequant_bf16_exact(rt):
    torch.manual_seed(4)
    x = (torch.randn(3000, 512) * 3).to(torch.bfloat16)
    pool = torch.zeros(4096, 288, dtype=torch.uint8, device="cuda")
    slots = torch.randperm(4096)[:3000]
    rt.write_nvfp4(x.cuda(), pool, slots.cuda())
    rows = torch.cat([slots[:1000], torch.tensor([-1, 5000])]).to(torch.int64)
    got = rt.dequant(pool, rows.cuda()).float().cpu().numpy()
    ref = O.dequant(pool.cpu().numpy(), rows.numpy())
    assert np.array_equal(got, ref)
    assert rt.device_errors() & 4          # row 5000 is outside the pool
