"""GPU: the rope side-pool (64 bf16 per token slot beside the 288-byte pool) through the C ABI.

The reference's model is NoPE: it drops k_pe at its write seam (nvfp4-kv/patch_nvfp4_kv.py:70)
and writes zero rope bytes into its 656-byte rows (nvfp4-kv/glm53_nvfp4_runtime.py:121-122).
The side-pool is this library's extension for MLA models that keep a rope part; the 288-byte
layout and every entry point without it are unchanged.  Checked here: the append copies k_pe
rows to their slots exactly; the 656-byte gather puts them in the fp8_ds_mla rope field byte for
byte; the fused decode adds q_rope . k_rope to the scores, against the oracle in float64 within
2e-2 relative / 1e-2 absolute elementwise and 1e-2 relative L2, and an all-zero side-pool gives
exactly the decode without one.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SM = 1.0 / 24.0
RTOL, ATOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def _pools(rt, pages, seed, rope_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(pages * 64, 512, generator=g).to(torch.bfloat16)
    pool_np = O.quant_new(x)
    pool = torch.from_numpy(pool_np).cuda().view(pages, 64, 288)
    k_pe = (torch.randn(pages * 64, 64, generator=g) * rope_scale).to(torch.bfloat16)
    rope = torch.zeros(pages, 64, 64, dtype=torch.bfloat16, device="cuda")
    rt.write_nvfp4_rope(k_pe.cuda(), rope, torch.arange(pages * 64, device="cuda"))
    rope_np = k_pe.view(torch.int16).numpy().view(np.uint16)
    return pool_np, pool, rope_np, rope


def _check(out, ref, what):
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all(), what
    rel = np.linalg.norm(o - ref) / max(np.linalg.norm(ref), 1e-30)
    close = np.isclose(o, ref, rtol=RTOL, atol=ATOL)
    assert close.all(), f"{what}: {int((~close).sum())} outside tolerance, rel L2 {rel:.3e}"
    assert rel < 1e-2, f"{what}: rel L2 {rel:.3e}"


def test_append_rope_copies_rows_to_slots(rt):
    g = torch.Generator().manual_seed(1)
    T, rows = 3000, 4096
    wide = torch.randn(T, 576, generator=g).to(torch.bfloat16)       # k_pe as the last 64 dims of a row
    slots = torch.randperm(rows, generator=g)[:T]
    slots[::37] = -1                                                  # skipped
    for k_pe in (wide[:, 512:], wide[:, 511:575]):                    # 16-byte aligned, and not
        rope = torch.zeros(rows, 64, dtype=torch.bfloat16, device="cuda")
        rt.write_nvfp4_rope(k_pe.cuda(), rope, slots.cuda())
        want = torch.zeros(rows, 64, dtype=torch.bfloat16)
        keep = slots >= 0
        want[slots[keep]] = k_pe[keep]
        assert torch.equal(rope.cpu().view(torch.int16), want.view(torch.int16))
    bad = slots.clone()
    bad[0] = rows + 5                                                 # past the pool: skipped, flagged
    rt.device_errors()
    rt.write_nvfp4_rope(wide[:, 512:].cuda(), torch.zeros(rows, 64, dtype=torch.bfloat16, device="cuda"), bad.cuda())
    assert rt.device_errors() & 2


def test_gather_ds656_rope_fills_the_rope_field(rt):
    pool_np, pool, rope_np, rope = _pools(rt, 64, seed=2)
    g = torch.Generator().manual_seed(3)
    idx = torch.randint(-2, 64 * 64 + 2, (5000,), dtype=torch.int32, generator=g)   # clamped ends
    out = torch.empty(5000, 656, dtype=torch.uint8, device="cuda")
    rt._gather(pool.view(-1, 288), idx.cuda(), out, rope=rope)
    ref = O.gather_ds656(pool_np, idx.numpy(), rope=rope_np)
    assert np.array_equal(out.cpu().numpy(), ref)
    plain = torch.empty_like(out)
    rt._gather(pool.view(-1, 288), idx.cuda(), plain)                  # without: zeros there
    assert np.array_equal(plain.cpu().numpy()[:, :528], ref[:, :528])
    assert not plain[:, 528:].any()


@pytest.mark.parametrize("lens,QL,H", [([4096, 1000, 129, 3000], 1, 64), ([2048, 777], 2, 64),
                                       ([600, 9000], 1, 128)])
def test_dense_decode_with_rope(rt, lens, QL, H):
    pool_np, pool, rope_np, rope = _pools(rt, 200, seed=sum(lens))
    g = torch.Generator().manual_seed(len(lens))
    B = len(lens)
    width = (max(lens) + 63) // 64
    tables = torch.stack([torch.randperm(200, generator=g)[:width] for _ in range(B)]).to(torch.int32)
    q = torch.randn(B, QL, H, 576, generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    out = rt.mla_decode(q.cuda(), pool, None, 128, 512, 64, tables.cuda(), sl.cuda(), max(lens),
                        bmm1_scale=SM, rope_cache=rope)
    ref = O.mla_decode(q.float(), pool_np, tables.numpy(), sl.numpy(), sparse=False, bmm1_scale=SM,
                       rope=rope_np)
    _check(out, ref, f"dense rope {lens} q_len {QL} heads {H}")
    norope = O.mla_decode(q.float(), pool_np, tables.numpy(), sl.numpy(), sparse=False, bmm1_scale=SM)
    assert np.abs(norope - ref).max() > 0.05                          # the rope part matters here
    assert rt.device_errors() == 0


def test_sparse_decode_with_rope(rt):
    pool_np, pool, rope_np, rope = _pools(rt, 256, seed=7)
    g = torch.Generator().manual_seed(8)
    B, topk = 6, 2048
    idx = torch.stack([torch.randperm(256 * 64, generator=g)[:topk] for _ in range(B)]).to(torch.int32)
    idx[torch.rand(B, topk, generator=g) < 0.1] = -1
    sl = torch.tensor([2048, 2000, 1, 1024, 0, 2048], dtype=torch.int32)
    q = torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16)
    out = rt.mla_decode(q.cuda(), pool, None, 128, 512, 64, idx.view(B, 1, topk).cuda(), sl.cuda(), topk,
                        sparse_mla_top_k=topk, bmm1_scale=SM, rope_cache=rope)
    ref = O.mla_decode(q.float(), pool_np, idx.view(B, 1, topk).numpy(), sl.numpy(), sparse=True,
                       bmm1_scale=SM, rope=rope_np)
    _check(out, ref, "sparse rope")
    assert rt.device_errors() == 0


def test_zero_rope_pool_equals_no_rope(rt):
    pool_np, pool, _, _ = _pools(rt, 128, seed=11)
    zero = torch.zeros(128, 64, 64, dtype=torch.bfloat16, device="cuda")
    g = torch.Generator().manual_seed(12)
    B = 4
    tables = torch.stack([torch.randperm(128, generator=g)[:64] for _ in range(B)]).to(torch.int32).cuda()
    sl = torch.tensor([4096, 3000, 50, 4000], dtype=torch.int32).cuda()
    q = torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16).cuda()
    a = rt.mla_decode(q, pool, None, 128, 512, 64, tables, sl, 4096, bmm1_scale=SM)
    b = rt.mla_decode(q, pool, None, 128, 512, 64, tables, sl, 4096, bmm1_scale=SM, rope_cache=zero)
    assert torch.equal(a, b)
