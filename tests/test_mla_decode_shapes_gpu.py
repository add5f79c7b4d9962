"""GPU: the fused decode over shapes the other decode tests do not reach, against the attention
oracle (float64 over the exactly dequantised pool), or, for the million-token context, against
a plain PyTorch fp32 reference on the GPU.

Covered: page sizes 16 / 32 / 128 / 256; 32 and 192 heads; MTP q_len 2, 4 and 8; q and out as
strided views with bmm2_scale != 1; a seq_len beyond max_seq_len (clamped, flagged); a
1,048,576-token context.  Tolerance as the other decode tests: 2e-2 relative / 1e-2 absolute
elementwise and a relative L2 below 1e-2.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SM = 1.0 / math.sqrt(576)


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def _check(rt, out, ref, what, errors_ok=0):
    err = rt.device_errors()
    assert err & ~errors_ok == 0, f"{what}: device error bits {err:#x}"
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all(), what
    rel = np.linalg.norm(o - ref) / max(np.linalg.norm(ref), 1e-30)
    close = np.isclose(o, ref, rtol=2e-2, atol=1e-2)
    assert close.all(), f"{what}: {int((~close).sum())} outside tolerance, rel L2 {rel:.3e}"
    assert rel < 1e-2, f"{what}: rel L2 {rel:.3e}"
    return err


def _case(rt, B, H, QL, lens, page, pages, seed, max_len=None, q=None, out=None, bmm2=1.0):
    g = torch.Generator().manual_seed(seed)
    pool_np = O.quant_new(torch.randn(pages * page, 512, generator=g).to(torch.bfloat16))
    pool = torch.from_numpy(pool_np).cuda().view(pages, page, 288)
    max_len = max_len or max(lens)
    width = (max_len + page - 1) // page
    tables = torch.stack([torch.randperm(pages, generator=g)[:width] for _ in range(B)]).to(torch.int32)
    if q is None:
        q = torch.randn(B, QL, H, 576, generator=g).to(torch.bfloat16).cuda()
    sl = torch.tensor(lens, dtype=torch.int32)
    res = rt.mla_decode(q, pool, None, 128, 512, 64, tables.cuda(), sl.cuda(), max_len, out=out,
                        bmm1_scale=SM, bmm2_scale=bmm2)
    ref = O.mla_decode(q.float().cpu(), pool_np, tables.numpy(), np.minimum(sl.numpy(), max_len),
                       sparse=False, page_size=page, bmm1_scale=SM, bmm2_scale=bmm2)
    return res, ref


@pytest.mark.parametrize("page", [16, 32, 128, 256])
def test_dense_page_sizes(rt, page):
    lens = [1000, 3333, 64, 129]
    pages = (4096 + page - 1) // page + 8
    out, ref = _case(rt, 4, 64, 1, lens, page, pages, seed=page)
    _check(rt, out, ref, f"page {page}")


@pytest.mark.parametrize("H,QL", [(32, 1), (192, 1), (64, 2), (64, 4), (16, 8)])
def test_dense_heads_and_mtp(rt, H, QL):
    out, ref = _case(rt, 3, H, QL, [1500, 7, 2600], 64, 48, seed=H * 10 + QL)
    _check(rt, out, ref, f"H {H} q_len {QL}")


def test_dense_strided_q_and_out_with_bmm2(rt):
    g = torch.Generator().manual_seed(77)
    B, H = 3, 64
    q_big = torch.randn(B, 1, H, 640, generator=g).to(torch.bfloat16).cuda()
    q = q_big[..., :576]                                   # head stride 640 elements
    out_big = torch.zeros(B, 1, H, 520, dtype=torch.bfloat16, device="cuda")
    out = out_big[..., :512]                               # head stride 520 elements
    res, ref = _case(rt, B, H, 1, [900, 2049, 33], 64, 40, seed=5, q=q, out=out, bmm2=0.5)
    assert res.data_ptr() == out.data_ptr()
    _check(rt, out, ref, "strided q / out, bmm2 0.5")
    assert torch.all(out_big[..., 512:] == 0), "writes stayed inside the rows"


def test_dense_seq_len_beyond_max_is_clamped_and_flagged(rt):
    out, ref = _case(rt, 2, 64, 1, [2000 + 300, 1500], 64, 40, seed=9, max_len=2000)
    err = _check(rt, out, ref, "clamped seq_len", errors_ok=16)
    assert err & 16, "NVFP4KV_DEVERR_SEQ_LEN not set"


def test_dense_one_million_token_context(rt):
    """1,048,576 tokens x 64 heads (16,384 pages): fp32 PyTorch reference over the exactly
    dequantised rows, in 64K-token chunks merged by log-sum-exp."""
    ctx, page, H = 1 << 20, 64, 64
    pages = ctx // page
    torch.manual_seed(4)
    pool = torch.empty(pages, page, 288, dtype=torch.uint8, device="cuda")
    for c in range(0, ctx, 1 << 18):
        rt.write_nvfp4(torch.randn(1 << 18, 512, device="cuda").to(torch.bfloat16), pool,
                       torch.arange(c, c + (1 << 18), device="cuda"))
    table = torch.randperm(pages, device="cuda").to(torch.int32).view(1, pages)
    q = torch.randn(1, 1, H, 576, device="cuda").to(torch.bfloat16)
    sl = torch.tensor([ctx], dtype=torch.int32, device="cuda")
    out, lse = rt.mla_decode_lse(q, pool, None, 128, 512, 64, table, sl, ctx, bmm1_scale=SM)
    assert rt.device_errors() == 0
    rows = (table[0].long().view(-1, 1) * page + torch.arange(page, device="cuda")).view(-1)
    qf = q[0, 0, :, :512].float()
    m = torch.full((H,), -float("inf"), device="cuda")
    den = torch.zeros(H, device="cuda")
    num = torch.zeros(H, 512, device="cuda")
    for c in range(0, ctx, 1 << 16):
        kv = rt.dequant(pool, rows[c:c + (1 << 16)]).float()          # exact values
        s = (qf @ kv.T) * SM                                          # [H, chunk]
        mc = torch.maximum(m, s.max(dim=1).values)
        a = torch.exp(m - mc)
        p = torch.exp(s - mc[:, None])
        den = den * a + p.sum(dim=1)
        num = num * a[:, None] + p @ kv
        m = mc
    ref = (num / den[:, None]).cpu().numpy()[None, None]
    ref_lse = (m + torch.log(den)).cpu().numpy()
    _check(rt, out, ref, "1M tokens")
    assert np.abs(lse[0, 0].cpu().numpy() - ref_lse).max() < 2e-3
