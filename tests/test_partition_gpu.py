"""GPU: the decode's log-sum-exp output (nvfp4kv_mla_decode_lse through the C ABI) against the
oracle, and the multi-GPU sequence partition run with the CUDA decode (ranks emulated one
after another on one GPU: each rank's units are decoded with mla_decode_lse, then merged).

Tolerances: lse within 2e-3 absolute (q is coded as four NVFP4 terms, relative error ~5e-5,
on scores of order 10); outputs as the decode tests (2e-2 relative / 1e-2 absolute).
"""
import math

import numpy as np
import pytest
import torch

from glm53_flash_dual_dgx_spark_b200 import partition as P
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SM = 1.0 / math.sqrt(576)
PAGE = 64


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def _pool(num_pages, seed):
    g = torch.Generator().manual_seed(seed)
    pool = O.quant_new(torch.randn(num_pages * PAGE, 512, generator=g).to(torch.bfloat16))
    return torch.from_numpy(pool).cuda().view(num_pages, PAGE, 288), pool


@pytest.mark.parametrize("B,H,QL,lens", [
    (40, 128, 1, None),                       # 80 query groups: one split per group
    (2, 64, 1, [5000, 777]),                  # many splits: lse from the combine kernel
    (3, 64, 3, [1000, 64, 2500]),             # causal MTP
])
def test_lse_matches_oracle(rt, B, H, QL, lens):
    pages = 96
    pool_t, pool = _pool(pages, seed=B + QL)
    g = torch.Generator().manual_seed(11)
    lens = lens or [int(x) for x in torch.randint(1, 4000, (B,), generator=g)]
    width = (max(lens) + PAGE - 1) // PAGE
    tables = torch.stack([torch.randperm(pages, generator=g)[:width] for _ in range(B)]).to(torch.int32)
    q = torch.randn(B, QL, H, 576, generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    out, lse = rt.mla_decode_lse(q.cuda(), pool_t, None, 128, 512, 64, tables.cuda(), sl.cuda(), max(lens),
                                 bmm1_scale=SM)
    assert rt.device_errors() == 0
    ref, ref_lse = O.mla_decode(q.float(), pool, tables.numpy(), sl.numpy(), sparse=False, bmm1_scale=SM,
                                return_lse=True)
    got = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.abs(got[fin] - ref_lse[fin]).max() < 2e-3
    assert np.allclose(out.float().cpu().numpy(), ref, rtol=2e-2, atol=1e-2)


def test_sparse_lse_matches_oracle(rt):
    pool_t, pool = _pool(128, seed=5)
    g = torch.Generator().manual_seed(3)
    B, K = 5, 1500
    idx = torch.randint(-1, 128 * PAGE, (B, 1, K), generator=g, dtype=torch.int32)
    sl = torch.tensor([1500, 1, 700, 0, 1499], dtype=torch.int32)
    q = torch.randn(B, 1, 64, 576, generator=g).to(torch.bfloat16)
    out, lse = rt.mla_decode_lse(q.cuda(), pool_t, None, 128, 512, 64, idx.cuda(), sl.cuda(), K,
                                 sparse_mla_top_k=K, bmm1_scale=SM)
    assert rt.device_errors() == 0
    ref, ref_lse = O.mla_decode(q.float(), pool, idx.numpy(), sl.numpy(), sparse=True, bmm1_scale=SM,
                                return_lse=True)
    got = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.abs(got[fin] - ref_lse[fin]).max() < 2e-3
    assert np.allclose(out.float().cpu().numpy(), ref, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("world,QL", [(3, 1), (4, 3)])
def test_partitioned_decode_matches_whole_sequences(rt, world, QL):
    lens = [3000, 128, 4500, 999]
    pages = sum((n + PAGE - 1) // PAGE for n in lens) + 4
    pool_t, pool = _pool(pages, seed=world)
    g = torch.Generator().manual_seed(world + 100)
    perm = torch.randperm(pages, generator=g).to(torch.int32)
    tables, k = [], 0
    for n in lens:
        m = (n + PAGE - 1) // PAGE
        tables.append(perm[k:k + m])
        k += m
    q = torch.randn(len(lens), QL, 64, 576, generator=g).to(torch.bfloat16).cuda()

    def decode_fn(qq, tb, sl, max_len):
        return rt.mla_decode_lse(qq, pool_t, None, 128, 512, 64, tb, sl, max_len, bmm1_scale=SM)

    plan = P.plan(lens, world, PAGE, q_len=QL)
    outs, lses, seqs = [], [], []
    for units in plan:                              # rank r's work, one rank after another
        if not units:
            continue
        ut = [tables[u.seq][u.start // PAGE:(u.end + PAGE - 1) // PAGE] for u in units]
        o, l = P.decode_units(decode_fn, q, units, ut)
        outs.append(o)
        lses.append(l)
        seqs += [u.seq for u in units]
    out, lse = P.merge(torch.cat(outs), torch.cat(lses), seqs, len(lens))
    assert rt.device_errors() == 0
    width = max(t.numel() for t in tables)
    tb = np.full((len(lens), width), -1, dtype=np.int32)
    for s, t in enumerate(tables):
        tb[s, :t.numel()] = t.numpy()
    ref, ref_lse = O.mla_decode(q.float().cpu(), pool, tb, np.array(lens), sparse=False, bmm1_scale=SM,
                                return_lse=True)
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 2e-3
    o = out.float().cpu().numpy()
    assert np.allclose(o, ref, rtol=2e-2, atol=1e-2)
    assert np.linalg.norm(o - ref) / np.linalg.norm(ref) < 1e-2
