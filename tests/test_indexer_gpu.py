"""GPU: the indexer K-pool (NVFP4 indexer keys) and the DSA top-k selection, through the C ABI.

The reference keeps its indexer keys in an fp8 pool (nvfp4-kv/PLAN.md:29) and notes that FP4
indexer keys need sm_100 (README.md:321); its selection is vLLM's DSA indexer, whose rule
(DeepSeek-V3.2's, vllm-0.22 model_executor/models/deepseek_v2.py:604-735) the oracle restates:
score[b, s] = sum_h w[b, h] * max(q[b, h] . k[s], 0) over visible positions, then the top-k.
Checked: the 72-byte key rows bit-exact against the oracle's quantisation (the latent rows'
rule); the scores against the oracle in float64; the selection exactly against the same rule
applied to the kernel's own fp32 scores (ascending positions, ties to the lowest), and its
overlap with the float64 selection; the selection feeding the sparse decode end to end.
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


def _keys(T, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(T, 128, generator=g)
    if outliers:
        k[torch.rand(T, 128, generator=g) < 0.01] *= 20
    return k.to(torch.bfloat16)


def test_index_append_bit_exact(rt):
    from test_append_edges_gpu import edge_rows
    for k in (_keys(5000, 1), edge_rows(torch.bfloat16)[:, :128].contiguous(),
              torch.cat([torch.zeros(3, 128), torch.full((2, 128), 1e-30)]).to(torch.bfloat16)):
        T = k.shape[0]
        rows = T + 17
        slots = torch.randperm(rows, generator=torch.Generator().manual_seed(T))[:T]
        slots[::29] = -1
        pool = torch.zeros(rows, 72, dtype=torch.uint8, device="cuda")
        rt.index_append(k.cuda(), pool, slots.cuda())
        want = np.zeros((rows, 72), np.uint8)
        keep = (slots >= 0).numpy()
        want[slots.numpy()[keep]] = O.index_quant(k)[keep]
        bad = np.argwhere(pool.cpu().numpy() != want)
        assert bad.size == 0, f"{len(bad)} bytes differ, first {bad[:6].tolist()}"
    wide = torch.randn(64, 576).to(torch.bfloat16)                      # a strided view
    pool = torch.zeros(64, 72, dtype=torch.uint8, device="cuda")
    rt.index_append(wide.cuda()[:, 200:328], pool, torch.arange(64, device="cuda"))
    assert np.array_equal(pool.cpu().numpy(), O.index_quant(wide[:, 200:328].contiguous()))
    assert rt.device_errors() == 0


def _case(rt, lens, pages, seed, topk=2048, missing=()):
    B = len(lens)
    pool_np = O.index_quant(_keys(pages * 64, seed))
    pool = torch.from_numpy(pool_np).cuda().view(pages, 64, 72)
    g = torch.Generator().manual_seed(seed + 1)
    width = (max(lens) + 63) // 64
    tables = torch.stack([torch.randperm(pages, generator=g)[:width] for _ in range(B)]).to(torch.int32)
    for b, j in missing:
        tables[b, j] = pages + 3                                        # a page outside the pool
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16)
    w = torch.rand(B, 64, generator=g) * 0.1
    sl = torch.tensor(lens, dtype=torch.int32)
    rows, counts = rt.index_topk(q.cuda(), w.cuda(), pool, tables.cuda(), sl.cuda(), max(lens), topk)
    torch.cuda.synchronize()
    ld = (max(lens) + 127) // 128 * 128
    gpu_scores = rt.index_scores_buffer()[:B * ld].view(B, ld).cpu().numpy()
    ref_scores = O.index_scores(q.float(), w, pool_np, tables.numpy(), lens)
    return pool_np, tables, q, w, sl, rows.cpu().numpy(), counts.cpu().numpy(), gpu_scores, ref_scores


@pytest.mark.parametrize("lens,missing", [([6000, 2048, 777, 4097], ()), ([9000, 3000], ((0, 5), (1, 2))),
                                          ([0, 3, 2049, 10000], ())])
def test_index_topk_scores_and_selection(rt, lens, missing):
    pages = 200
    pool_np, tables, q, w, sl, rows, counts, gs, rs = _case(rt, lens, pages, seed=sum(lens), missing=missing)
    topk = 2048
    for b, n in enumerate(lens):
        if n == 0:                                                      # nothing visible: no rows
            assert counts[b] == 0 and (rows[b] == -1).all()
            continue
        ref = rs[b]
        got = gs[b, :n]
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(got), fin)
        assert np.allclose(got[fin], ref[fin], rtol=1e-4, atol=1e-4 * np.abs(ref[fin]).max())
        assert counts[b] == min(n, topk)
        # the selection rule applied to the kernel's own scores: exact
        pos = O.index_select(got.astype(np.float64), topk)
        pg = tables[b].numpy()[pos // 64].astype(np.int64)
        want = np.where((pg >= 0) & (pg < pages), pg * 64 + pos % 64, -1)
        assert np.array_equal(rows[b, :len(pos)], want), f"entry {b}: selection differs"
        assert (rows[b, len(pos):] == -1).all()
        # against the float64 selection: only near-ties at the threshold may differ
        exact = set(O.index_select(ref, topk).tolist())
        assert len(exact & set(pos.tolist())) >= 0.995 * len(pos)
    assert rt.device_errors() == 0


def test_index_topk_ties_go_to_lowest_positions(rt):
    pages = 64
    k = torch.full((pages * 64, 128), 0.5).to(torch.bfloat16)            # every score equal
    pool = torch.from_numpy(O.index_quant(k)).cuda().view(pages, 64, 72)
    tables = torch.arange(pages, dtype=torch.int32).view(1, pages).cuda()
    q = torch.ones(1, 64, 128).to(torch.bfloat16).cuda()
    w = torch.ones(1, 64).cuda()
    sl = torch.tensor([4000], dtype=torch.int32).cuda()
    rows, counts = rt.index_topk(q, w, pool, tables, sl, 4000, 2048)
    assert int(counts[0]) == 2048
    assert torch.equal(rows[0].cpu(), torch.arange(2048, dtype=torch.int32))


def test_index_topk_feeds_the_sparse_decode(rt):
    """The DSA read path end to end: NVFP4 indexer keys -> top-2048 rows -> fused sparse decode
    over the 288-byte latent pool, against the oracle on the same rows."""
    pages = 160
    lens = [8000, 1500, 5000]
    pool_np, tables, _, _, sl, _, _, _, _ = _case(rt, lens, pages, seed=5)
    g = torch.Generator().manual_seed(6)
    latent = torch.randn(pages * 64, 512, generator=g).to(torch.bfloat16)
    kv_np = O.quant_new(latent)
    kv = torch.from_numpy(kv_np).cuda().view(pages, 64, 288)
    iq = torch.randn(3, 64, 128, generator=g).to(torch.bfloat16).cuda()
    iw = (torch.rand(3, 64, generator=g) * 0.1).cuda()
    index = torch.from_numpy(pool_np).cuda().view(pages, 64, 72)
    rows, counts = rt.index_topk(iq, iw, index, tables.cuda(), sl.cuda(), max(lens), 2048)
    q = torch.randn(3, 1, 64, 576, generator=g).to(torch.bfloat16)
    out = rt.mla_decode(q.cuda(), kv, None, 128, 512, 64, rows.view(3, 1, 2048), counts, 2048,
                        sparse_mla_top_k=2048, bmm1_scale=1.0 / 24)
    ref = O.mla_decode(q.float(), kv_np, rows.cpu().view(3, 1, 2048).numpy(), counts.cpu().numpy(), sparse=True,
                       bmm1_scale=1.0 / 24)
    o = out.float().cpu().numpy()
    assert np.allclose(o, ref, rtol=2e-2, atol=1e-2)
    assert np.linalg.norm(o - ref) / np.linalg.norm(ref) < 1e-2
    assert rt.device_errors() == 0


def test_index_topk_long_runs_wrap_every_ring(rt):
    """16 entries of 16K positions: each score block takes about 15 key tiles, so the key ring
    and the operand, accumulator and loader rings all wrap several times.  The scores and the
    selection are checked as above, and a call must end promptly: a ring that stalls shows up
    as bounded waits running to their limit, not as an error."""
    import time
    lens = [16384] * 16
    pages = 16 * 256
    pool_np, tables, q, w, sl, rows, counts, gs, rs = _case(rt, lens, pages, seed=11)
    for b, n in enumerate(lens):
        ref, got = rs[b], gs[b, :n]
        assert np.allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
        pos = O.index_select(got.astype(np.float64), 2048)
        pg = tables[b].numpy()[pos // 64].astype(np.int64)
        assert np.array_equal(rows[b, :len(pos)], pg * 64 + pos % 64)
    pool = torch.from_numpy(pool_np).cuda().view(pages, 64, 72)
    args = (q.cuda(), w.cuda(), pool, tables.cuda(), sl.cuda(), max(lens), 2048)
    rt.index_topk(*args)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(3):
        rt.index_topk(*args)
    torch.cuda.synchronize()
    assert time.perf_counter() - t < 0.3, "index_topk took seconds: a pipeline wait ran to its limit"
    assert rt.device_errors() == 0
    for _ in range(200):                      # a rare stall still sets the timeout bit
        rt.index_topk(*args)
    torch.cuda.synchronize()
    assert rt.device_errors() == 0


@pytest.mark.parametrize("page", [2, 16, 256])
def test_index_topk_other_page_sizes(rt, page):
    """The scoring kernel copies a tile of 128 keys as 128 / page whole pages (2 and 16 rows) or
    as a 128-row run inside one page (256 rows); sequence ends fall inside a tile and inside a
    page, and one page is missing."""
    lens = [3001, 777, 1500]
    pages = (4096 + page - 1) // page * 2
    pool_np = O.index_quant(_keys(pages * page, seed=page))
    pool = torch.from_numpy(pool_np).cuda().view(pages, page, 72)
    g = torch.Generator().manual_seed(page + 1)
    width = (max(lens) + page - 1) // page
    tables = torch.stack([torch.randperm(pages, generator=g)[:width] for _ in lens]).to(torch.int32)
    tables[0, width // 2] = pages + 5                                   # a page outside the pool
    q = torch.randn(len(lens), 64, 128, generator=g).to(torch.bfloat16)
    w = torch.rand(len(lens), 64, generator=g) * 0.1
    topk = 512
    rows, counts = rt.index_topk(q.cuda(), w.cuda(), pool, tables.cuda(), torch.tensor(lens, dtype=torch.int32).cuda(),
                                 max(lens), topk)
    torch.cuda.synchronize()
    ld = (max(lens) + 127) // 128 * 128
    gs = rt.index_scores_buffer()[:len(lens) * ld].view(len(lens), ld).cpu().numpy()
    rs = O.index_scores(q.float(), w, pool_np, tables.numpy(), lens, page_size=page)
    rows, counts = rows.cpu().numpy(), counts.cpu().numpy()
    for b, n in enumerate(lens):
        ref, got = rs[b], gs[b, :n]
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(got), fin)
        assert np.allclose(got[fin], ref[fin], rtol=1e-4, atol=1e-4 * np.abs(ref[fin]).max())
        assert counts[b] == min(n, topk)
        pos = O.index_select(got.astype(np.float64), topk)
        pg = tables[b].numpy()[pos // page].astype(np.int64)
        want = np.where((pg >= 0) & (pg < pages), pg * page + pos % page, -1)
        assert np.array_equal(rows[b, :len(pos)], want), f"page {page}, entry {b}: selection differs"
    assert rt.device_errors() == 0
