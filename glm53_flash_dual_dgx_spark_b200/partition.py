"""Multi-GPU sequence partition for the NVFP4 MLA decode: one process per GPU.

The decode shards without a data-path collective: every sequence's pages are independent, so
a rank owns the pool pages of its work units, appends into them and attends them locally.  A
work unit is a page-aligned token range of one sequence.  ``plan`` lays the batch's tokens
end to end and cuts that stream into ``world_size`` page-aligned ranges of (nearly) equal
token counts.  Every rank gets the same work ±1 page, and a sequence is split only where a
cut falls inside it.

Results of the pieces of one sequence merge exactly through the log-sum-exp of each piece
(``merge``): out = sum_r exp(lse_r - L) out_r with L = log sum_r exp(lse_r).  The only
collective is one all-gather of the per-unit (out, lse) after the decode (``gather_merge``).

Causal MTP (q_len > 1): query token i sees tokens t < seq_len - (q_len - 1 - i).  A piece that
ends before the sequence's last q_len - 1 tokens is therefore visible to every query token:
it is decoded with q_len folded into the heads (``decode_units``), a free view of q.  The
last piece of a sequence is decoded as usual, so the kernel applies the causal limit at its
end.  The cuts are page-aligned and a last piece holds at least one page, so a last piece
always contains the final q_len - 1 tokens when q_len - 1 <= page_size.

The reference's KV path runs on one GPU and has no counterpart of this module; it is the
multi-GPU form of the same decode (sequence plus page-range units, token-balanced, merged
by log-sum-exp).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch


@dataclass(frozen=True)
class Unit:
    """Tokens [start, end) of sequence ``seq``; ``last`` when end is the sequence's end."""
    seq: int
    start: int
    end: int
    last: bool

    @property
    def tokens(self) -> int:
        return self.end - self.start


def plan(seq_lens: Sequence[int], world_size: int, page_size: int = 64, q_len: int = 1) -> list[list[Unit]]:
    """Token-balanced assignment of page-aligned sequence pieces to ``world_size`` ranks.

    The sequences are laid end to end in batch order; the stream is cut into ``world_size``
    ranges whose boundaries are the page-aligned points closest to k * total / world_size
    (within each sequence: a cut never leaves a piece of less than one page at a sequence's
    end).  Deterministic: every rank computes the same plan.  Empty sequences produce no unit.
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    if page_size < 1 or q_len < 1:
        raise ValueError("page_size and q_len must be >= 1")
    if q_len - 1 > page_size:
        raise ValueError("q_len - 1 must not exceed page_size (the last piece holds the causal tail)")
    lens = [int(x) for x in seq_lens]
    if any(x < 0 for x in lens):
        raise ValueError("negative sequence length")
    total = sum(lens)
    # candidate cut points: page boundaries inside sequences (never within the final page),
    # plus sequence boundaries, in stream coordinates
    cuts = [0]
    base = 0
    for n in lens:
        last_page_start = ((n - 1) // page_size) * page_size if n > 0 else 0
        for off in range(page_size, last_page_start + 1, page_size):
            cuts.append(base + off)
        base += n
        cuts.append(base)
    cuts = sorted(set(cuts))
    # rank r takes the stream range [b_r, b_{r+1}); b_r = the candidate closest to r * total / W
    bounds = [0]
    j = 0
    for r in range(1, world_size):
        target = r * total / world_size
        while j + 1 < len(cuts) and abs(cuts[j + 1] - target) <= abs(cuts[j] - target):
            j += 1
        bounds.append(max(cuts[j], bounds[-1]))
    bounds.append(total)
    out: list[list[Unit]] = [[] for _ in range(world_size)]
    starts = []
    base = 0
    for n in lens:
        starts.append(base)
        base += n
    for r in range(world_size):
        lo, hi = bounds[r], bounds[r + 1]
        for s, n in enumerate(lens):
            a, b = max(lo, starts[s]), min(hi, starts[s] + n)
            if a < b:
                out[r].append(Unit(s, a - starts[s], b - starts[s], b - starts[s] == n))
    return out


def rank_tokens(units: Sequence[Unit]) -> int:
    return sum(u.tokens for u in units)


DecodeFn = Callable[..., tuple]
"""decode_fn(q [B, QL, H, D], tables [B, W] int32, seq_lens [B] int32, max_seq_len) ->
(out [B, QL, H, 512], lse [B, QL, H] float32): the rank-local decode (the CUDA path wraps
glm53_nvfp4_runtime.mla_decode_lse)."""


def decode_units(decode_fn: DecodeFn, q: torch.Tensor, units: Sequence[Unit],
                 tables: Sequence[torch.Tensor]):
    """Decode this rank's units; ``tables[k]`` lists unit k's local page ids (its pages in the
    rank-local pool, in token order).  q is the batch's query [B, QL, H, D] (every rank holds
    all of it: it is small).  Returns (out [U, QL, H, 512], lse [U, QL, H] float32) in unit
    order.  Non-last units run as one call with q_len folded into the heads; last units as
    one call with the causal limit."""
    B, QL, H, D = q.shape
    U = len(units)
    dev = q.device
    out = torch.empty(U, QL, H, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(U, QL, H, dtype=torch.float32, device=dev)
    for last in (False, True):
        idx = [k for k, u in enumerate(units) if u.last == last]
        if not idx:
            continue
        width = max(tables[k].numel() for k in idx)
        tb = torch.full((len(idx), max(width, 1)), -1, dtype=torch.int32, device=dev)
        for row, k in enumerate(idx):
            tb[row, :tables[k].numel()] = tables[k].to(device=dev, dtype=torch.int32)
        sl = torch.tensor([units[k].tokens for k in idx], dtype=torch.int32, device=dev)
        qs = q[[units[k].seq for k in idx]].contiguous()
        if not last and QL > 1:
            o, l = decode_fn(qs.view(len(idx), 1, QL * H, D), tb, sl, int(sl.max()))
            o, l = o.view(len(idx), QL, H, 512), l.view(len(idx), QL, H)
        else:
            o, l = decode_fn(qs, tb, sl, int(sl.max()))
        out[idx] = o.to(out.dtype)
        lse[idx] = l.float()
    return out, lse


def merge(parts_out: torch.Tensor, parts_lse: torch.Tensor, seq_of_part: Sequence[int], batch: int):
    """Merge per-piece results into per-sequence results.

    parts_out [P, QL, H, 512], parts_lse [P, QL, H]; ``seq_of_part[p]`` is piece p's sequence
    (a list, or a long tensor on the parts' device).
    Returns (out [batch, QL, H, 512] in parts_out's dtype, lse [batch, QL, H] float32);
    a row no piece sees (every lse -inf, or no piece at all) is zeros with lse -inf."""
    P, QL, H, D = parts_out.shape
    dev = parts_out.device
    # a device index tensor keeps the merge free of host copies (CUDA-graph capturable)
    seq = (seq_of_part.to(device=dev, dtype=torch.long) if torch.is_tensor(seq_of_part)
           else torch.as_tensor(list(seq_of_part), dtype=torch.long, device=dev))
    lse = torch.full((batch, QL, H), float("-inf"), dtype=torch.float32, device=dev)
    if P:
        lse = lse.scatter_reduce(0, seq.view(-1, 1, 1).expand(P, QL, H), parts_lse.float(), "amax",
                                 include_self=True)
    m = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    w = torch.exp(parts_lse.float() - m[seq])                     # 0 for a piece with lse -inf
    den = torch.zeros(batch, QL, H, dtype=torch.float32, device=dev).index_add(0, seq, w)
    num = torch.zeros(batch, QL, H, D, dtype=torch.float32, device=dev).index_add(
        0, seq, w.unsqueeze(-1) * parts_out.float())
    out = torch.where(den.unsqueeze(-1) > 0, num / den.clamp_min(1e-30).unsqueeze(-1), torch.zeros_like(num))
    lse = torch.where(den > 0, m + torch.log(den.clamp_min(1e-30)), torch.full_like(den, float("-inf")))
    return out.to(parts_out.dtype), lse


def gather_merge(out_u: torch.Tensor, lse_u: torch.Tensor, plan_: Sequence[Sequence[Unit]], rank: int,
                 batch: int, group=None):
    """All-gather every rank's unit results (the one collective) and merge them into the
    batch's output on every rank.  ``plan_`` is ``plan``'s result (identical on all ranks);
    ``out_u``/``lse_u`` are this rank's ``decode_units`` results.  Ranks with fewer units pad."""
    import torch.distributed as dist
    world = len(plan_)
    assert len(plan_[rank]) == out_u.shape[0]
    umax = max(1, max(len(u) for u in plan_))
    QL, H, D = out_u.shape[1:]
    po = torch.zeros(umax, QL, H, D, dtype=out_u.dtype, device=out_u.device)
    pl = torch.full((umax, QL, H), float("-inf"), dtype=torch.float32, device=out_u.device)
    po[:out_u.shape[0]] = out_u
    pl[:lse_u.shape[0]] = lse_u
    go = [torch.empty_like(po) for _ in range(world)]
    gl = [torch.empty_like(pl) for _ in range(world)]
    dist.all_gather(go, po, group=group)
    dist.all_gather(gl, pl, group=group)
    outs, lses, seqs = [], [], []
    for r in range(world):
        n = len(plan_[r])
        outs.append(go[r][:n])
        lses.append(gl[r][:n])
        seqs += [u.seq for u in plan_[r]]
    return merge(torch.cat(outs), torch.cat(lses), seqs, batch)
