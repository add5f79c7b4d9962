"""CPU: the multi-GPU sequence partition (glm53_flash_dual_dgx_spark_b200/partition.py).

The rank-local decode is the attention oracle here (float64 over the exactly dequantised pool,
returning the log-sum-exp too), injected as ``decode_fn``; the GPU test of the same flow with
the CUDA kernel is in test_partition_gpu.py.  Checked: the plan covers every token once,
page-aligned, balanced to a page; merging the pieces of split sequences reproduces the whole
-sequence result (dense, and causal MTP with q_len 3); and the same through a real
two-process gloo all-gather.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from glm53_flash_dual_dgx_spark_b200 import partition as P
from oracle import oracle as O

SM = 1.0 / math.sqrt(576)
PAGE = 64


@pytest.mark.parametrize("lens,world", [
    ([8192] * 16, 1), ([8192] * 16, 3), ([460000] * 5 + [900000] * 3, 8),
    ([100, 0, 5000, 70], 4), ([64], 4), ([1000, 3], 2), ([129, 64, 65], 5),
])
def test_plan_covers_every_token_once_balanced(lens, world):
    plan = P.plan(lens, world, PAGE)
    assert len(plan) == world
    pieces = {}
    for units in plan:
        for u in units:
            assert 0 <= u.start < u.end <= lens[u.seq]
            assert u.start % PAGE == 0
            assert u.last == (u.end == lens[u.seq])
            pieces.setdefault(u.seq, []).append((u.start, u.end))
    for s, n in enumerate(lens):
        got = sorted(pieces.get(s, []))
        if n == 0:
            assert not got
            continue
        assert got[0][0] == 0 and got[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(got, got[1:])), got
        assert n - got[-1][0] >= min(n, 1)
    loads = [P.rank_tokens(u) for u in plan]
    assert sum(loads) == sum(lens)
    if sum(lens) >= world * PAGE * 4:
        assert max(loads) - min(loads) <= PAGE, loads
    assert P.plan(lens, world, PAGE) == plan            # deterministic


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        P.plan([10], 0)
    with pytest.raises(ValueError):
        P.plan([-1], 2)
    with pytest.raises(ValueError):
        P.plan([10], 2, page_size=16, q_len=18)


def _problem(B=4, H=64, QL=1, lens=(1000, 2048, 333, 1600), seed=0):
    g = torch.Generator().manual_seed(seed)
    pages_per = [(n + PAGE - 1) // PAGE for n in lens]
    num_pages = sum(pages_per) + 3
    pool = O.quant_new(torch.randn(num_pages * PAGE, 512, generator=g).to(torch.bfloat16))
    perm = torch.randperm(num_pages, generator=g)
    tables, k = [], 0
    for n in pages_per:
        tables.append(perm[k:k + n].to(torch.int32))
        k += n
    q = torch.randn(B, QL, H, 576, generator=g).to(torch.bfloat16)
    return pool, tables, q, list(lens)


def _oracle_fn(pool):
    def fn(q, tables, seq_lens, max_seq_len):
        out, lse = O.mla_decode(q.float(), pool, tables.numpy(), seq_lens.numpy(), sparse=False,
                                page_size=PAGE, bmm1_scale=SM, return_lse=True)
        return torch.from_numpy(out).float(), torch.from_numpy(lse).float()
    return fn


def _unit_tables(units, tables):
    return [tables[u.seq][u.start // PAGE:(u.end + PAGE - 1) // PAGE] for u in units]


def _full(pool, tables, q, lens):
    width = max(t.numel() for t in tables)
    tb = np.full((len(lens), width), -1, dtype=np.int32)
    for s, t in enumerate(tables):
        tb[s, :t.numel()] = t.numpy()
    return O.mla_decode(q.float(), pool, tb, np.array(lens, dtype=np.int32), sparse=False,
                        page_size=PAGE, bmm1_scale=SM, return_lse=True)


@pytest.mark.parametrize("world,QL", [(1, 1), (3, 1), (5, 1), (4, 3)])
def test_pieces_merge_to_the_whole_sequence_result(world, QL):
    pool, tables, q, lens = _problem(QL=QL, seed=world * 10 + QL)
    plan = P.plan(lens, world, PAGE, q_len=QL)
    fn = _oracle_fn(pool)
    outs, lses, seqs = [], [], []
    for units in plan:
        if not units:
            continue
        o, l = P.decode_units(fn, q, units, _unit_tables(units, tables))
        outs.append(o)
        lses.append(l)
        seqs += [u.seq for u in units]
    out, lse = P.merge(torch.cat(outs), torch.cat(lses), seqs, len(lens))
    ref, ref_lse = _full(pool, tables, q, lens)
    assert np.allclose(lse.numpy(), ref_lse, rtol=1e-5, atol=1e-4)
    assert np.allclose(out.float().numpy(), ref, rtol=2e-2, atol=1e-2)
    rel = np.linalg.norm(out.float().numpy() - ref) / np.linalg.norm(ref)
    assert rel < 1e-2, rel


def test_merge_rows_without_tokens():
    out = torch.randn(3, 1, 2, 512)
    lse = torch.tensor([[[0.5, float("-inf")]], [[1.0, float("-inf")]], [[float("-inf"), float("-inf")]]])
    m, ml = P.merge(out, lse, [0, 0, 1], 3)
    w = torch.softmax(torch.tensor([0.5, 1.0]), 0)
    assert torch.allclose(m[0, 0, 0], w[0] * out[0, 0, 0] + w[1] * out[1, 0, 0], atol=1e-6)
    assert torch.all(m[0, 0, 1] == 0) and ml[0, 0, 1] == float("-inf")
    assert torch.all(m[1] == 0) and torch.all(m[2] == 0)           # no visible token / no piece
    assert torch.isinf(ml[2]).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pool, tables, q, lens = _problem(QL=3, seed=7)
        plan = P.plan(lens, world, PAGE, q_len=3)
        units = plan[rank]
        o, l = P.decode_units(_oracle_fn(pool), q, units, _unit_tables(units, tables))
        out, lse = P.gather_merge(o, l, plan, rank, len(lens))
        if rank == 0:
            ref, ref_lse = _full(pool, tables, q, lens)
            ok = bool(np.allclose(out.float().numpy(), ref, rtol=2e-2, atol=1e-2)
                      and np.allclose(lse.numpy(), ref_lse, rtol=1e-5, atol=1e-4))
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_gather_merge_over_two_gloo_ranks(tmp_path):
    result = tmp_path / "result.txt"
    mp.start_processes(_gloo_rank, args=(2, _free_port(), str(result)), nprocs=2, join=True,
                       start_method="spawn")
    assert result.read_text() == "ok"
