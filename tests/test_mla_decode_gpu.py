"""GPU: the fused NVFP4 gather + MLA decode kernel (C ABI via the drop-in mla_decode) against
the attention oracle (float64 softmax(q K^T * s) V over the exactly dequantised pool rows).

Tolerance: bf16 output within 2e-2 relative / 1e-2 absolute of the
oracle, elementwise (torch.allclose(rtol=2e-2, atol=1e-2)).  The kernel is additionally held
to a relative L2 error below 1e-2, which is what fp16 probabilities and a bf16 output allow.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL, REL_L2 = 2e-2, 1e-2, 1e-2
SM = 1.0 / math.sqrt(576)


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def make_pool(num_pages, page=64, seed=0, scale=1.0, device="cuda"):
    """Random N(0,1) latent quantised by the oracle (CPU), uploaded."""
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(num_pages * page, 512, generator=g) * scale).to(torch.bfloat16)
    pool = O.quant_new(x)
    return torch.from_numpy(pool).to(device).view(num_pages, page, 288), pool


def check(out, ref, what="", errors_ok=0):
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    err = rt.device_errors()
    assert err & ~errors_ok == 0, f"{what}: device error bits {err:#x}"
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all(), f"{what}: non-finite output"
    rel = np.linalg.norm(o - ref) / max(np.linalg.norm(ref), 1e-30)
    close = np.isclose(o, ref, rtol=RTOL, atol=ATOL)
    assert close.all(), f"{what}: {int((~close).sum())} elements outside tolerance, rel L2 {rel:.3e}"
    assert rel < REL_L2, f"{what}: rel L2 {rel:.3e}"
    return rel


def run_dense(rt, B, H, QL, seq_lens, num_pages=64, page=64, seed=0, qscale=1.0, kvscale=1.0):
    pool_t, pool = make_pool(num_pages, page, seed, kvscale)
    g = torch.Generator().manual_seed(seed + 1)
    max_len = max(max(seq_lens), 1)
    width = (max_len + page - 1) // page
    tables = torch.stack([torch.randperm(num_pages, generator=g)[:width] for _ in range(B)]).to(torch.int32)
    q = (torch.randn(B, QL, H, 576, generator=g) * qscale).to(torch.bfloat16)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, tables.cuda(), sl.cuda(), max_len,
                        bmm1_scale=SM, bmm2_scale=1.0)
    ref = O.mla_decode(q.float(), pool, tables.numpy(), sl.numpy(), sparse=False, page_size=page,
                       bmm1_scale=SM)
    return out, ref


@pytest.mark.parametrize("seq_lens", [[1], [127, 128, 129], [300, 1, 64, 1000], [4096]])
def test_dense_ragged_lengths(rt, seq_lens):
    out, ref = run_dense(rt, len(seq_lens), 64, 1, seq_lens)
    check(out, ref, f"dense {seq_lens}")
    assert rt.device_errors() == 0


def test_dense_16_heads_padded_rows(rt):
    """H=16 as in the reference's test_kernel_equiv.py (16 real rows of the 64-row tile)."""
    out, ref = run_dense(rt, 5, 16, 1, [2048, 700, 33, 1500, 129])
    check(out, ref, "H=16")


def test_dense_128_heads_two_groups(rt):
    out, ref = run_dense(rt, 2, 128, 1, [515, 2000])
    check(out, ref, "H=128")


def test_dense_mtp_causal(rt):
    """q_len 3 (MTP): query token i sees seq_len - (2 - i) tokens."""
    out, ref = run_dense(rt, 3, 64, 3, [130, 2, 1000])
    check(out, ref, "MTP")


def test_dense_peaked_softmax_rescales(rt):
    """Large logits make the running max move by far more than the lazy-rescale threshold."""
    out, ref = run_dense(rt, 2, 64, 1, [3000, 1024], qscale=8.0)
    check(out, ref, "peaked")


def test_dense_many_tiles_per_split(rt):
    """20 x 128 heads = 40 work units: 3 splits of 11 tiles each, so every CTA walks its raw-tile
    ring several times over and carries O across tiles."""
    out, ref = run_dense(rt, 20, 128, 1, [4000 - 97 * k for k in range(20)], num_pages=64)
    check(out, ref, "many tiles")


def test_dense_many_tiles_peaked(rt):
    """Multi-tile CTAs with large logits: the running max moves across tiles and O^T is rescaled."""
    out, ref = run_dense(rt, 20, 64, 1, [3000] * 10 + [2500] * 10, num_pages=48, qscale=8.0)
    check(out, ref, "many tiles peaked")


def test_dense_zero_length_and_bad_page(rt):
    pool_t, pool = make_pool(16)
    q = torch.randn(3, 1, 64, 576).to(torch.bfloat16)
    tables = torch.tensor([[0, 1, 2], [3, 99, 5], [6, 7, 8]], dtype=torch.int32)   # page 99 invalid
    sl = torch.tensor([0, 150, 100], dtype=torch.int32)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, tables.cuda(), sl.cuda(), 192, bmm1_scale=SM)
    o = out.float().cpu().numpy()
    assert (o[0] == 0).all()
    assert rt.device_errors() & 8
    # entry 1: tokens on page 99 are masked -> same as attending tokens 0-63 and 128-149
    ref1 = O.mla_decode(q[1:2].float(), pool, np.array([[3, 99, 5]]), np.array([150]), sparse=False,
                        bmm1_scale=SM)
    rows = np.concatenate([3 * 64 + np.arange(64), 5 * 64 + np.arange(22)])
    kv = O.dequant(pool, rows).astype(np.float64)
    s = q[1, 0, :, :512].double().numpy() @ kv.T * SM
    p = np.exp(s - s.max(1, keepdims=True))
    manual = (p / p.sum(1, keepdims=True)) @ kv
    assert np.allclose(ref1[0, 0], manual)
    check(out[1:2], manual[None, None], "masked page")
    check(out[2:3], O.mla_decode(q[2:3].float(), pool, tables[2:3].numpy(), np.array([100]), sparse=False,
                                 bmm1_scale=SM), "entry 2")


def test_dense_config2_full_size(rt):
    """Config 2: batch 16, 64 heads, qk 576, v 512, 8K context, page table = randperm(2048)."""
    torch.manual_seed(0)
    B, H, ctx, pages = 16, 64, 8192, 2048
    x = torch.randn(pages * 64, 512).to(torch.bfloat16)
    pool_np = np.zeros((pages * 64, 288), np.uint8)
    O.quant(x, np.arange(pages * 64), pool_np)
    tables = torch.randperm(pages).to(torch.int32).view(B, ctx // 64)
    q = torch.randn(B, 1, H, 576).to(torch.bfloat16)
    sl = torch.full((B,), ctx, dtype=torch.int32)
    pool_t = torch.from_numpy(pool_np).cuda().view(pages, 64, 288)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, tables.cuda(), sl.cuda(), ctx, bmm1_scale=SM)
    ref = O.mla_decode(q.float(), pool_np, tables.numpy(), sl.numpy(), sparse=False, bmm1_scale=SM)
    check(out, ref, "config 2")


@pytest.mark.parametrize("topk,pad", [(2048, 0.0), (2048, 0.1), (333, 0.05)])
def test_sparse_topk(rt, topk, pad):
    """Sparse (indexer) decode: per-query top-k physical rows, -1 padded, seq_lens = counts."""
    pool_t, pool = make_pool(512, seed=3)
    R = 512 * 64
    g = torch.Generator().manual_seed(1)
    B = 6
    idx = torch.stack([torch.randperm(R, generator=g)[:topk] for _ in range(B)]).to(torch.int32)
    idx[torch.rand(B, topk, generator=g) < pad] = -1
    sl = torch.tensor([topk, topk - 7, 1, topk // 2, 0, topk], dtype=torch.int32)
    q = torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, idx.view(B, 1, topk).cuda(), sl.cuda(), topk,
                        sparse_mla_top_k=topk, bmm1_scale=SM)
    ref = O.mla_decode(q.float(), pool, idx.view(B, 1, topk).numpy(), sl.numpy(), sparse=True, bmm1_scale=SM)
    check(out, ref, f"sparse topk={topk} pad={pad}")
    assert rt.device_errors() == 0


def run_sparse(rt, B, H, topk, seq_lens, seed=5, qscale=1.0, pool_pages=256, bad=0.0, pad=0.0, QL=1):
    pool_t, pool = make_pool(pool_pages, seed=seed)
    R = pool_pages * 64
    g = torch.Generator().manual_seed(seed + 1)
    # rows drawn with replacement: repeated rows are legal top-k entries
    idx = torch.randint(0, R, (B, topk), generator=g, dtype=torch.int32)
    idx[torch.rand(B, topk, generator=g) < pad] = -1
    nbad = torch.rand(B, topk, generator=g) < bad
    idx[nbad] = torch.where(torch.rand(B, topk, generator=g) < 0.5, R + 17, -5).to(torch.int32)[nbad]
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    q = (torch.randn(B, QL, H, 576, generator=g) * qscale).to(torch.bfloat16)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, idx.view(B, 1, topk).cuda(), sl.cuda(), topk,
                        sparse_mla_top_k=topk, bmm1_scale=SM)
    ref = O.mla_decode(q.float(), pool, idx.view(B, 1, topk).numpy(), sl.numpy(), sparse=True, bmm1_scale=SM)
    return out, ref


def test_sparse_many_tiles_per_split(rt):
    """20 entries x 128 heads = 40 query groups: 3 splits of ~11 tiles each, so the 3-slot
    tile ring wraps many times and each split's ~1365 row ids exceed the 768 staged in
    shared memory (the one-row-per-lane copy path); ragged counts end tiles mid-way."""
    out, ref = run_sparse(rt, 20, 128, 4096, [4096, 4000, 3001, 129] * 5)
    check(out, ref, "sparse many tiles")


def test_sparse_prefill_tokens_one_split_each(rt):
    """A prefill step through the sparse path: 160 query tokens of one sequence, each with its
    own top-2048 rows from a causal window (a window grows by one row per token), so every
    query group is its own CTA (no split) with 16 tiles, and its 2048 row ids stream through
    the 768-entry window the load warp refills ahead of its copies.  Eight tokens are checked
    against the oracle."""
    pool_t, pool = make_pool(320, seed=31)
    R = 320 * 64
    g = torch.Generator().manual_seed(32)
    T, topk, prior = 160, 2048, 16000
    idx = torch.empty(T, topk, dtype=torch.int32)
    for i in range(T):
        idx[i] = torch.randperm(prior + i + 1, generator=g)[:topk].to(torch.int32)
    perm = torch.randperm(R, generator=g).to(torch.int32)       # positions -> shuffled pool rows
    idx = perm[idx.long()]
    sl = torch.full((T,), topk, dtype=torch.int32)
    sl[5] = 2000                                                  # one ragged count
    q = torch.randn(T, 1, 64, 576, generator=g).to(torch.bfloat16)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, idx.view(T, 1, topk).cuda(), sl.cuda(), topk,
                        sparse_mla_top_k=topk, bmm1_scale=SM)
    pick = [0, 5, 37, 64, 99, 128, 150, 159]
    ref = O.mla_decode(q[pick].float(), pool, idx[pick].view(len(pick), 1, topk).numpy(), sl[pick].numpy(),
                       sparse=True, bmm1_scale=SM)
    check(out[pick], ref, "sparse prefill tokens")
    assert rt.device_errors() == 0


def test_sparse_peaked_scores(rt):
    out, ref = run_sparse(rt, 8, 64, 2048, [2048] * 4 + [1500] * 4, qscale=8.0, seed=11)
    check(out, ref, "sparse peaked")


def test_sparse_rejects_multi_token_queries(rt):
    """Sparse top-k tables hold one list per batch entry; a multi-token query (MTP) has one
    top-k set per token, so callers pass tokens as batch entries.  q_len > 1 is refused."""
    from glm53_flash_dual_dgx_spark_b200 import _lib
    with pytest.raises(_lib.Nvfp4kvError, match="q_len == 1"):
        run_sparse(rt, 2, 64, 256, [256, 100], QL=2)


def test_sparse_out_of_range_indices_masked(rt):
    """Entries < -1 or >= pool_rows are masked like -1 padding and flag BAD_INDEX."""
    out, ref = run_sparse(rt, 6, 64, 1024, [1024, 1000, 700, 1024, 5, 1024], bad=0.05, pad=0.05, seed=21)
    check(out, ref, "sparse bad indices", errors_ok=4)


def test_sparse_config3_shape(rt):
    """Config 3 at full size: batch 16, 64 heads, 128K context per sequence (pool of
    2,097,152 rows on shuffled pages), top-2048 drawn without replacement (seed 1)."""
    B, ctx, topk = 16, 131072, 2048
    pages = B * ctx // 64
    torch.manual_seed(0)
    pool_t = torch.empty(pages, 64, 288, dtype=torch.uint8, device="cuda")
    for c in range(0, pages * 64, 1 << 20):                     # quantise on the GPU in chunks
        n = min(1 << 20, pages * 64 - c)
        x = torch.randn(n, 512, device="cuda").to(torch.bfloat16)
        rt.write_nvfp4(x, pool_t, torch.arange(c, c + n, device="cuda"))
    page_table = torch.randperm(pages).view(B, ctx // 64)
    torch.manual_seed(1)
    logical = torch.stack([torch.randperm(ctx)[:topk] for _ in range(B)])
    phys = (page_table.gather(1, logical // 64) * 64 + logical % 64).to(torch.int32)
    q = torch.randn(B, 1, 64, 576).to(torch.bfloat16)
    sl = torch.full((B,), topk, dtype=torch.int32)
    out = rt.mla_decode(q.cuda(), pool_t, None, 128, 512, 64, phys.view(B, 1, topk).cuda(), sl.cuda(), topk,
                        sparse_mla_top_k=topk, bmm1_scale=SM)
    rows = phys.view(-1).long().cuda()
    sub = pool_t.view(-1, 288)[rows].cpu().numpy()               # only the rows the oracle needs
    local = np.arange(B * topk, dtype=np.int32).reshape(B, 1, topk)
    ref = O.mla_decode(q.float(), sub, local, sl.numpy(), sparse=True, bmm1_scale=SM)
    check(out, ref, "config 3")


def test_cuda_graph_replay_matches_eager(rt):
    pool_t, pool = make_pool(64)
    g = torch.Generator().manual_seed(7)
    B = 4
    tables = torch.stack([torch.randperm(64, generator=g)[:32] for _ in range(B)]).to(torch.int32).cuda()
    sl = torch.tensor([2048, 100, 1500, 777], dtype=torch.int32).cuda()
    q = torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16).cuda()
    out = torch.empty(B, 1, 64, 512, dtype=torch.bfloat16, device="cuda")
    rt.mla_decode(q, pool_t, None, 128, 512, 64, tables, sl, 2048, out=out, bmm1_scale=SM)  # warm-up
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            rt.mla_decode(q, pool_t, None, 128, 512, 64, tables, sl, 2048, out=out, bmm1_scale=SM)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    q.copy_(torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16))
    graph.replay()
    ref = O.mla_decode(q.float().cpu(), pool, tables.cpu().numpy(), sl.cpu().numpy(), sparse=False, bmm1_scale=SM)
    check(out, ref, "graph replay")
