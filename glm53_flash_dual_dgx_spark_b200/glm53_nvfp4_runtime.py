"""Drop-in NVFP4 KV-pool runtime for B200 (sm_100a).

Same module surface as the reference's ``nvfp4-kv/glm53_nvfp4_runtime.py``
(Plaaasma/glm53-flash-dual-dgx-spark), which the vLLM seam patcher copies into the vLLM
package as ``vllm.glm53_nvfp4_runtime``:

    NV_BYTES, DS_BYTES, enabled(), write_nvfp4(), _gather(), build_scratch(),
    _SYNC_FREE_T, _bufs

plus the fused read path the reference does not have:

    mla_decode(query, kv_cache, workspace_buffer, qk_nope_head_dim, kv_lora_rank,
               qk_rope_head_dim, block_tables, seq_lens, max_seq_len,
               sparse_mla_top_k=0, out=None, bmm1_scale=1.0, bmm2_scale=1.0)

argument-compatible with FlashInfer's ``trtllm_batch_decode_with_kv_cache_mla`` (the
consumer the reference feeds, patch_nvfp4_kv.py:84-118) but reading the 288-byte pool
rows directly instead of a 656-byte fp8 scratch.

Every compute call goes through the C ABI of ``libnvfp4kv.so`` on the current torch CUDA
stream; nothing synchronises the host and nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

NV_BYTES = 288
DS_BYTES = 656
LATENT = 512
ROPE = 64

_ON = os.environ.get("GLM53_NVFP4_KV", "0") == "1"          # read once at import (runtime:29)

# Sync-free ceiling of build_scratch (runtime:134-140): steps with at most this many query
# tokens gather every table entry into a persistent buffer (no host sync, graph-safe).
_SYNC_FREE_T = int(os.environ.get("GLM53_NVFP4_SYNCFREE_T", "192"))
# The T > _SYNC_FREE_T branch of build_scratch deduplicates on the device
# (build_scratch_sync_free), so no step synchronises the host.  GLM53_NVFP4_UNIQUE=1 restores
# the reference's torch.unique branch (runtime:177-182), which synchronises to size its output.
_UNIQUE = os.environ.get("GLM53_NVFP4_UNIQUE", "0") == "1"
# Rows of the device branch's persistent scratch (656 B each).  0 (default): min(T * K, pool
# rows + 1), the most distinct entries a step can have; a smaller bound caps the memory, and a
# step with more distinct entries than it sets NVFP4KV_DEVERR_CAPACITY.
_SYNC_FREE_ROWS = int(os.environ.get("GLM53_NVFP4_SYNCFREE_ROWS", "0"))

# Division of the 656 B row encoders (_gather, build_scratch): "ieee" (default) gives the
# reference's rows as it computes on the CPU, "triton" its rows as Triton compiles it for the
# GPU (approximate fp32 division), byte for byte.  See set_gather_division.
_GATHER_DIV = os.environ.get("GLM53_NVFP4_GATHER_DIV", "ieee")

# Persistent device buffers keyed like the reference's: ("shared", K, device index) for the
# build_scratch buffer; ("err", index) / ("ws", index) for this module's own state.
_bufs: dict = {}
_ws_sizes: dict = {}   # decode workspace bytes per (batch, q_len, heads, max_seq_len, topk, device)


def enabled() -> bool:
    return _ON


# ------------------------------------------------------------------ helpers
def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this runtime has no CPU path)")


def _err_word(dev: torch.device) -> torch.Tensor:
    key = ("err", dev.index)
    e = _bufs.get(key)
    if e is None:
        e = torch.zeros(1, dtype=torch.int32, device=dev)
        _bufs[key] = e
    return e


def device_errors(device=None, clear: bool = True) -> int:
    """Read (and by default clear) the device error word: OR of NVFP4KV_DEVERR_* bits.

    Synchronises with the device; meant for tests and health checks, not the hot path.
    """
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    e = _err_word(dev)
    v = int(e.item())
    if clear:
        e.zero_()
    return v


class _on_device:
    """Make `dev` current for the C call when it is not already (launches use it)."""

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev.index:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# ------------------------------------------------------------------ write path
def write_nvfp4(kv_c: torch.Tensor, kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """kv_c [T, 512] -> NVFP4 rows at slot_mapping in kv_cache (viewed [-1, 288]).

    Same contract as the reference (runtime:68-76): T == 0 is a no-op, slots < 0 are
    skipped.  Slots past the pool are skipped too and flagged in the device error word.
    """
    pool = kv_cache.view(-1, NV_BYTES)
    T = kv_c.shape[0]
    if T == 0:
        return
    _require_cuda(kv_c, "kv_c")
    _require_cuda(pool, "kv_cache")
    if kv_c.dtype == torch.bfloat16:
        dt = _lib.DTYPE_BF16
    elif kv_c.dtype == torch.float16:
        dt = _lib.DTYPE_F16
    else:
        raise TypeError(f"kv_c must be bfloat16 or float16, got {kv_c.dtype}")
    if kv_c.dim() != 2 or kv_c.shape[1] < LATENT or kv_c.stride(1) != 1:
        raise ValueError("kv_c must be [T, >=512] with a contiguous last dimension")
    if pool.dtype != torch.uint8:
        raise TypeError("kv_cache must be a uint8 pool")
    slot = slot_mapping.reshape(-1)
    if slot.numel() != T:
        raise ValueError(f"slot_mapping has {slot.numel()} entries for {T} tokens")
    if slot.dtype == torch.int64:
        sdt = _lib.INDEX_I64
    elif slot.dtype == torch.int32:
        sdt = _lib.INDEX_I32
    else:
        raise TypeError("slot_mapping must be int64 or int32")
    slot = slot.contiguous()
    dev = kv_c.device
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_append(kv_c.data_ptr(), dt, T, kv_c.stride(0), pool.data_ptr(),
                                       pool.shape[0], slot.data_ptr(), sdt,
                                       _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_append")


def write_nvfp4_rope(k_pe: torch.Tensor, rope_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """k_pe [T, 64] bf16 -> the rope side-pool rope_cache (any shape, 64 bf16 per token slot) at
    slot_mapping; slots < 0 are skipped.  Not in the reference, which drops k_pe for its NoPE
    model (patch_nvfp4_kv.py:70); for MLA models that keep a rope part, beside write_nvfp4."""
    T = k_pe.shape[0]
    if T == 0:
        return
    _require_cuda(k_pe, "k_pe")
    _require_cuda(rope_cache, "rope_cache")
    if k_pe.dtype != torch.bfloat16 or k_pe.dim() != 2 or k_pe.shape[1] < ROPE or k_pe.stride(1) != 1:
        raise ValueError("k_pe must be bf16 [T, >=64] with a contiguous last dimension")
    rope = rope_cache.view(-1, ROPE)
    if rope.dtype != torch.bfloat16:
        raise TypeError("rope_cache must be bf16")
    slot = slot_mapping.reshape(-1).contiguous()
    if slot.numel() != T:
        raise ValueError(f"slot_mapping has {slot.numel()} entries for {T} tokens")
    sdt = _lib.INDEX_I64 if slot.dtype == torch.int64 else _lib.INDEX_I32 if slot.dtype == torch.int32 else None
    if sdt is None:
        raise TypeError("slot_mapping must be int64 or int32")
    dev = k_pe.device
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_append_rope(k_pe.data_ptr(), T, k_pe.stride(0), rope.data_ptr(), rope.shape[0],
                                            slot.data_ptr(), sdt, _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_append_rope")


# ------------------------------------------------------------------ 656-byte read path
def set_gather_division(mode: str) -> None:
    """Division of the 656-byte row encoders, process-wide: "ieee" (exact; the reference's
    _gather_kernel as it computes on the CPU) or "triton" (div.full.f32, the approximate fp32
    division GPU Triton compiles the reference's `amax / 448.0` and `1.0 / gscale` to, so the
    rows are byte-identical to the reference's GPU output).  No counterpart in the reference."""
    modes = {"ieee": _lib.DIV_IEEE, "triton": _lib.DIV_TRITON}
    if mode not in modes:
        raise ValueError(f"gather division must be 'ieee' or 'triton', got {mode!r}")
    _lib.check(_lib.lib().nvfp4kv_set_gather_division(modes[mode]), "nvfp4kv_set_gather_division")


def get_gather_division() -> str:
    return "triton" if _lib.lib().nvfp4kv_get_gather_division() == _lib.DIV_TRITON else "ieee"


if _GATHER_DIV != "ieee":
    set_gather_division(_GATHER_DIV)


def _gather(pool: torch.Tensor, idx: torch.Tensor, out: torch.Tensor, rope: torch.Tensor | None = None) -> None:
    """NVFP4 pool rows at idx -> fp8_ds_mla 656-byte rows in out (runtime:128-131).  With a rope
    side-pool ``rope`` (not in the reference) the rows' rope bytes carry its 64 bf16."""
    S = idx.shape[0]
    if S == 0:
        return
    _require_cuda(pool, "pool")
    if idx.dtype != torch.int32:
        raise TypeError("idx must be int32")
    if out.dtype != torch.uint8 or out.shape[-1] != DS_BYTES or not out.is_contiguous():
        raise ValueError("out must be a contiguous [S, 656] uint8 tensor")
    idx = idx.contiguous()
    dev = pool.device
    with _on_device(dev):
        if rope is None:
            rc = _lib.lib().nvfp4kv_gather_ds656(pool.data_ptr(), pool.shape[0], idx.data_ptr(), S,
                                                 out.data_ptr(), _stream(dev))
        else:
            r = rope.reshape(-1, ROPE)
            if r.dtype != torch.bfloat16 or r.shape[0] != pool.shape[0] or not r.is_contiguous():
                raise ValueError("rope must be a contiguous bf16 [pool rows, 64] side-pool")
            rc = _lib.lib().nvfp4kv_gather_ds656_rope(pool.data_ptr(), r.data_ptr(), pool.shape[0], idx.data_ptr(),
                                                      S, out.data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_gather_ds656")


def build_scratch(kv_cache: torch.Tensor, block_tables: torch.Tensor):
    """kv_cache: allocated pool (any shape, 288 B/token rows).
    block_tables: [T, 1, K] int32 physical token rows (-1 padded).
    Returns (scratch [P, 64, 656] uint8, tables [T, 1, K] into scratch), as the reference
    (runtime:143-182): T <= _SYNC_FREE_T gathers every entry into a persistent buffer with
    fixed shapes and no host sync.  Larger T deduplicates on the device without a host sync
    (build_scratch_sync_free): the tables equal the reference's, and the reference's
    ceil(n_unique / 64) pages are the first pages of a persistent capacity-sized scratch (the
    consumer reads only the rows the tables name).  With GLM53_NVFP4_UNIQUE=1 the large branch
    is the reference's torch.unique one, which synchronises the host.
    """
    pool = kv_cache.view(-1, NV_BYTES)
    T, one, K = block_tables.shape
    flat = block_tables.view(-1)
    dev = pool.device
    if T <= _SYNC_FREE_T:
        S = T * K
        P = (S + 63) // 64
        key = ("shared", K, dev.index)
        ent = _bufs.get(key)
        if ent is None:
            pcap = (_SYNC_FREE_T * K + 63) // 64
            ent = (torch.zeros(pcap, 64, DS_BYTES, dtype=torch.uint8, device=dev),
                   torch.arange(pcap * 64, dtype=torch.int32, device=dev))
            _bufs[key] = ent
        buf, ar = ent
        _gather(pool, flat, buf.view(-1, DS_BYTES)[:S])
        return buf[:P], ar[:S].view(T, 1, K)
    if not _UNIQUE:
        scratch, tables, _ = build_scratch_sync_free(kv_cache, block_tables,
                                                     capacity_rows=_SYNC_FREE_ROWS or None)
        return scratch, tables
    uniq, inv = torch.unique(flat, return_inverse=True)
    S = uniq.shape[0]
    P = (S + 63) // 64
    scratch = torch.zeros(P, 64, DS_BYTES, dtype=torch.uint8, device=dev)
    _gather(pool, uniq.to(torch.int32), scratch.view(-1, DS_BYTES)[:S])
    return scratch, inv.to(torch.int32).view(T, 1, K)


def build_scratch_sync_free(kv_cache: torch.Tensor, block_tables: torch.Tensor,
                            capacity_rows: int | None = None):
    """The T > _SYNC_FREE_T branch of build_scratch without a host synchronisation.

    The reference deduplicates with torch.unique (runtime:177-182), which synchronises to
    size its output.  Here the distinct entries are found, numbered in ascending order and
    gathered on the device by fixed-size launches (nvfp4kv_dedup_gather_ds656), so the call
    is asynchronous and CUDA-graph capturable.  Returns (scratch [P_cap, 64, 656] uint8,
    tables [T, 1, K] int32, n_unique int32 [1] on the device).  tables equals the
    reference's; the reference's scratch is the first ceil(n_unique / 64) pages of this one
    (rows from n_unique to the end of that page are zero); later pages are not written.
    P_cap covers capacity_rows rows, by default min(T * K, pool rows + 1), the most distinct
    entries there can be; fewer rows than the distinct entries set NVFP4KV_DEVERR_CAPACITY.
    The scratch is a view of one persistent buffer per device, allocated when a call needs
    more rows than it holds (656 B per row; for a 2,713,846-row pool and 2048 x 2048 entries
    the default capacity is 2,713,847 rows = 1.78 GB) and overwritten by the next call, like
    the reference's persistent sync-free buffer.
    """
    pool = kv_cache.view(-1, NV_BYTES)
    _require_cuda(pool, "kv_cache")
    _require_cuda(block_tables, "block_tables")
    if block_tables.dim() != 3:
        raise ValueError("block_tables must be [T, 1, K]")
    if block_tables.dtype != torch.int32:
        raise TypeError("block_tables must be int32")
    T, one, K = block_tables.shape
    flat = block_tables.reshape(-1).contiguous()
    n = flat.numel()
    R = pool.shape[0]
    cap = min(n, R + 1) if capacity_rows is None else int(capacity_rows)
    if cap < 0:
        raise ValueError("capacity_rows must be >= 0")
    dev = pool.device
    P = (cap + 63) // 64
    skey = ("dedup_scratch", dev.index)
    buf = _bufs.get(skey)
    if buf is None or buf.shape[0] < P:
        _bufs.pop(skey, None)
        buf = torch.empty(P, 64, DS_BYTES, dtype=torch.uint8, device=dev)
        _bufs[skey] = buf
    scratch = buf[:P]
    tables = torch.empty(n, dtype=torch.int32, device=dev)
    n_unique = torch.empty(1, dtype=torch.int32, device=dev)
    ints = ctypes.c_int64()
    _lib.check(_lib.lib().nvfp4kv_dedup_workspace_ints(R, n, ctypes.byref(ints)), "nvfp4kv_dedup_workspace_ints")
    key = ("dedup", dev.index)
    ws = _bufs.get(key)
    if ws is None or ws.numel() < ints.value:
        ws = torch.empty(ints.value, dtype=torch.int32, device=dev)
        _bufs[key] = ws
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_dedup_gather_ds656(pool.data_ptr(), R, flat.data_ptr(), n, ws.data_ptr(),
                                                   ws.numel(), tables.data_ptr(), scratch.data_ptr(), P * 64,
                                                   n_unique.data_ptr(), _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_dedup_gather_ds656")
    return scratch, tables.view(T, 1, K), n_unique


def dequant(kv_cache: torch.Tensor, rows: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Pool rows -> bf16 [n, 512] (exact); rows outside the pool (and -1) read as zeros."""
    pool = kv_cache.view(-1, NV_BYTES)
    rows = rows.reshape(-1)
    n = rows.numel()
    if out is None:
        out = torch.empty(n, LATENT, dtype=torch.bfloat16, device=pool.device)
    if n == 0:
        return out
    _require_cuda(pool, "kv_cache")
    if rows.dtype == torch.int64:
        rdt = _lib.INDEX_I64
    elif rows.dtype == torch.int32:
        rdt = _lib.INDEX_I32
    else:
        raise TypeError("rows must be int64 or int32")
    if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() < n * LATENT:
        raise ValueError("out must be a contiguous bf16 [n, 512] tensor")
    rows = rows.contiguous()
    dev = pool.device
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_dequant_bf16(pool.data_ptr(), pool.shape[0], rows.data_ptr(), rdt, n,
                                             out.data_ptr(), _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_dequant_bf16")
    return out


# ------------------------------------------------------------------ fused read path
def mla_decode_workspace_size(batch: int, q_len: int, num_heads: int, max_seq_len: int,
                              sparse_mla_top_k: int = 0, device=None) -> int:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = ctypes.c_size_t(0)
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_mla_decode_workspace_size(batch, q_len, num_heads, max_seq_len,
                                                          sparse_mla_top_k, ctypes.byref(out))
    _lib.check(rc, "nvfp4kv_mla_decode_workspace_size")
    return int(out.value)


def mla_decode_plan(batch: int, q_len: int, num_heads: int, max_seq_len: int,
                    sparse_mla_top_k: int = 0, device=None) -> tuple[int, int]:
    """(token splits per 64-row query group, kernel launches per mla_decode call)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    splits, launches = ctypes.c_int(0), ctypes.c_int(0)
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_mla_decode_plan(batch, q_len, num_heads, max_seq_len, sparse_mla_top_k,
                                                ctypes.byref(splits), ctypes.byref(launches))
    _lib.check(rc, "nvfp4kv_mla_decode_plan")
    return int(splits.value), int(launches.value)


def set_kernel_events(start: torch.cuda.Event | None, stop: torch.cuda.Event | None) -> None:
    """Make the calling thread's next mla_decode record `start` / `stop` immediately around its
    attention kernel (a measurement hook; both None clears it)."""
    for e in (start, stop):
        if e is not None and not e.cuda_event:
            e.record()   # torch creates the CUDA event on first record; the library re-records it
    _lib.check(_lib.lib().nvfp4kv_set_kernel_events(
        ctypes.c_void_p(start.cuda_event) if start is not None else None,
        ctypes.c_void_p(stop.cuda_event) if stop is not None else None), "nvfp4kv_set_kernel_events")


def _workspace(dev: torch.device, nbytes: int, given: torch.Tensor | None) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    if given is not None and given.is_cuda and given.numel() * given.element_size() >= nbytes \
            and given.data_ptr() % 256 == 0 and given.is_contiguous():
        return given
    key = ("ws", dev.index)
    ws = _bufs.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _bufs[key] = ws
    return ws


def mla_decode(query: torch.Tensor, kv_cache: torch.Tensor, workspace_buffer: torch.Tensor | None,
               qk_nope_head_dim: int, kv_lora_rank: int, qk_rope_head_dim: int,
               block_tables: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int,
               sparse_mla_top_k: int = 0, out: torch.Tensor | None = None,
               bmm1_scale: float = 1.0, bmm2_scale: float = 1.0,
               rope_cache: torch.Tensor | None = None) -> torch.Tensor:
    """Fused NVFP4 gather + MLA decode (see module docstring).

    query: [B, q_len, H, kv_lora_rank + qk_rope_head_dim] bf16.
    kv_cache: the 288-byte pool, [num_pages, page_size, 288] (or [num_pages, 1, page_size,
      288]); page_size is read from dim -2.
    Dense (sparse_mla_top_k == 0): block_tables [B, max_pages] page ids, seq_lens = context
      lengths.  Sparse: block_tables [B, 1, K] or [B, K] physical token rows (-1 padded),
      seq_lens = number of leading entries to use.
    Returns out [B, q_len, H, kv_lora_rank] bf16.  ``workspace_buffer`` is used for the
    split partials when it is large enough, else a persistent per-device buffer is.
    rope_cache (not in the reference, whose model is NoPE): the rope side-pool, [num_pages,
    page_size, 64] bf16 written by write_nvfp4_rope; the query's last 64 dims then meet it.
    """
    del qk_nope_head_dim  # accepted for signature compatibility; the absorbed MLA form ignores it
    return _decode(query, kv_cache, workspace_buffer, kv_lora_rank, qk_rope_head_dim, block_tables,
                   seq_lens, max_seq_len, sparse_mla_top_k, out, bmm1_scale, bmm2_scale, None, rope_cache)


def mla_decode_lse(query: torch.Tensor, kv_cache: torch.Tensor, workspace_buffer: torch.Tensor | None,
                   qk_nope_head_dim: int, kv_lora_rank: int, qk_rope_head_dim: int,
                   block_tables: torch.Tensor, seq_lens: torch.Tensor, max_seq_len: int,
                   sparse_mla_top_k: int = 0, out: torch.Tensor | None = None,
                   bmm1_scale: float = 1.0, bmm2_scale: float = 1.0):
    """mla_decode that also returns lse [B, q_len, H] float32: the natural log of the sum over
    the visible tokens of exp(bmm1_scale * q.k) (-inf for a row that sees no token).  Results of
    disjoint token ranges of one sequence merge exactly through it (see ``partition``).
    Returns (out, lse).  No counterpart in the reference; used by the multi-GPU partition."""
    del qk_nope_head_dim
    B, QL, H = query.shape[0], query.shape[1], query.shape[2]
    lse = torch.empty(B, QL, H, dtype=torch.float32, device=query.device)
    out = _decode(query, kv_cache, workspace_buffer, kv_lora_rank, qk_rope_head_dim, block_tables,
                  seq_lens, max_seq_len, sparse_mla_top_k, out, bmm1_scale, bmm2_scale, lse)
    return out, lse


def _decode(query, kv_cache, workspace_buffer, kv_lora_rank, qk_rope_head_dim, block_tables,
            seq_lens, max_seq_len, sparse_mla_top_k, out, bmm1_scale, bmm2_scale, lse, rope_cache=None):
    _require_cuda(query, "query")
    _require_cuda(kv_cache, "kv_cache")
    if isinstance(bmm1_scale, torch.Tensor) or isinstance(bmm2_scale, torch.Tensor):
        raise TypeError("bmm1_scale / bmm2_scale must be Python floats (a device scalar would need a sync)")
    if query.dtype != torch.bfloat16 or query.dim() != 4:
        raise ValueError("query must be a 4-D bf16 tensor [B, q_len, H, D]")
    if query.stride(3) != 1:
        raise ValueError("query's last dimension must be contiguous")
    B, QL, H, D = query.shape
    if kv_lora_rank != LATENT or D != kv_lora_rank + qk_rope_head_dim:
        raise ValueError(f"query dim {D} must equal kv_lora_rank (512) + qk_rope_head_dim")
    pool = kv_cache.view(-1, NV_BYTES)
    page_size = kv_cache.shape[-2] if kv_cache.dim() >= 3 else 64
    sparse = int(sparse_mla_top_k) > 0
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_tables and seq_lens must be int32")
    bt = block_tables.reshape(B, -1) if sparse else block_tables
    if bt.dim() != 2 or bt.stride(1) != 1:
        raise ValueError("block_tables must be [B, width] with a contiguous last dimension")
    if sparse and bt.shape[1] < sparse_mla_top_k:
        raise ValueError("sparse block_tables narrower than sparse_mla_top_k")
    if not sparse and bt.shape[1] * page_size < max_seq_len:
        raise ValueError("block_tables too narrow for max_seq_len")
    sl = seq_lens.contiguous()
    if out is None:
        out = torch.empty(B, QL, H, LATENT, dtype=torch.bfloat16, device=query.device)
    elif out.shape != (B, QL, H, LATENT) or out.dtype != torch.bfloat16 or out.stride(3) != 1:
        raise ValueError("out must be bf16 [B, q_len, H, 512] with a contiguous last dimension")
    rope = None
    if rope_cache is not None:
        if lse is not None:
            raise ValueError("mla_decode_lse has no rope variant")
        _require_cuda(rope_cache, "rope_cache")
        rope = rope_cache.reshape(-1, ROPE)
        if rope.dtype != torch.bfloat16 or rope.shape[0] != pool.shape[0] or not rope.is_contiguous():
            raise ValueError("rope_cache must be a contiguous bf16 [pool rows, 64] side-pool")
    dev = query.device
    with _on_device(dev):
        size_key = (B, QL, H, int(max_seq_len), int(sparse_mla_top_k), dev.index, rope is not None)
        ws_need = _ws_sizes.get(size_key)
        if ws_need is None:                      # the plan depends only on these and the device
            if rope is None:
                ws_need = mla_decode_workspace_size(B, QL, H, max_seq_len, int(sparse_mla_top_k), dev)
            else:
                n = ctypes.c_size_t(0)
                _lib.check(_lib.lib().nvfp4kv_mla_decode_rope_workspace_size(
                    B, QL, H, int(max_seq_len), int(sparse_mla_top_k), ctypes.byref(n)),
                    "nvfp4kv_mla_decode_rope_workspace_size")
                ws_need = int(n.value)
            _ws_sizes[size_key] = ws_need
        ws = _workspace(dev, ws_need, workspace_buffer)
        args = [query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
                pool.data_ptr(), pool.shape[0],
                bt.data_ptr(), bt.stride(0), sl.data_ptr(),
                B, QL, H, D, kv_lora_rank,
                int(sparse_mla_top_k), int(page_size), int(max_seq_len),
                float(bmm1_scale), float(bmm2_scale),
                out.data_ptr(), out.stride(0), out.stride(1), out.stride(2)]
        tail = [ws.data_ptr() if ws is not None else None, ws_need, _err_word(dev).data_ptr(), _stream(dev)]
        if rope is not None:
            rc = _lib.lib().nvfp4kv_mla_decode_rope(*args[:6], rope.data_ptr(), *args[6:], *tail)
        elif lse is None:
            rc = _lib.lib().nvfp4kv_mla_decode(*args, *tail)
        else:
            rc = _lib.lib().nvfp4kv_mla_decode_lse(*args, lse.data_ptr(), *tail)
    _lib.check(rc, "nvfp4kv_mla_decode")
    return out


# ------------------------------------------------------------------ indexer K-pool
INDEX_DIM = 128
INDEX_ROW_BYTES = 72


def index_append(k: torch.Tensor, index_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Indexer keys k [T, 128] bf16 -> NVFP4 72-byte rows of index_cache (any shape, 72 bytes per
    token slot) at slot_mapping; slots < 0 are skipped.  The reference keeps its indexer keys in
    an fp8 pool (PLAN.md:29); this is the FP4 pool its README (:321) leaves to sm_100."""
    T = k.shape[0]
    if T == 0:
        return
    _require_cuda(k, "k")
    _require_cuda(index_cache, "index_cache")
    if k.dtype != torch.bfloat16 or k.dim() != 2 or k.shape[1] < INDEX_DIM or k.stride(1) != 1:
        raise ValueError("k must be bf16 [T, >=128] with a contiguous last dimension")
    pool = index_cache.view(-1, INDEX_ROW_BYTES)
    if pool.dtype != torch.uint8:
        raise TypeError("index_cache must be uint8")
    slot = slot_mapping.reshape(-1).contiguous()
    if slot.numel() != T:
        raise ValueError(f"slot_mapping has {slot.numel()} entries for {T} tokens")
    sdt = _lib.INDEX_I64 if slot.dtype == torch.int64 else _lib.INDEX_I32 if slot.dtype == torch.int32 else None
    if sdt is None:
        raise TypeError("slot_mapping must be int64 or int32")
    dev = k.device
    with _on_device(dev):
        rc = _lib.lib().nvfp4kv_index_append(k.data_ptr(), T, k.stride(0), pool.data_ptr(), pool.shape[0],
                                             slot.data_ptr(), sdt, _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_index_append")


def index_topk(q: torch.Tensor, weights: torch.Tensor, index_cache: torch.Tensor, block_tables: torch.Tensor,
               seq_lens: torch.Tensor, max_seq_len: int, topk: int = 2048,
               out_rows: torch.Tensor | None = None, out_count: torch.Tensor | None = None):
    """The DSA indexer's selection over the NVFP4 indexer pool: per entry b, the pool rows of the
    topk positions s < seq_lens[b] with the highest sum_h weights[b, h] * max(q[b, h] . k[s], 0),
    in ascending position order (-1 padded), and their count min(seq_lens[b], topk).
    q [B, 64, 128] bf16, weights [B, 64] fp32, block_tables [B, pages] page ids.  The two
    results are the sparse tables and seq_lens mla_decode(..., sparse_mla_top_k=topk) takes.
    No host synchronisation; the score workspace is a persistent per-device buffer."""
    _require_cuda(q, "q")
    B = q.shape[0]
    if q.dtype != torch.bfloat16 or q.dim() != 3 or q.shape[2] != INDEX_DIM or q.stride(2) != 1:
        raise ValueError("q must be bf16 [B, 64, 128] with a contiguous last dimension")
    if weights.dtype != torch.float32 or weights.shape[0] != B or weights.stride(1) != 1:
        raise ValueError("weights must be float32 [B, 64]")
    pool = index_cache.view(-1, INDEX_ROW_BYTES)
    page_size = index_cache.shape[-2] if index_cache.dim() >= 3 else 64
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_tables and seq_lens must be int32")
    dev = q.device
    if out_rows is None:
        out_rows = torch.empty(B, topk, dtype=torch.int32, device=dev)
    if out_count is None:
        out_count = torch.empty(B, dtype=torch.int32, device=dev)
    with _on_device(dev):
        need = ctypes.c_size_t(0)
        _lib.check(_lib.lib().nvfp4kv_index_topk_workspace_size(B, int(max_seq_len), ctypes.byref(need)),
                   "nvfp4kv_index_topk_workspace_size")
        key = ("index_ws", dev.index)
        ws = _bufs.get(key)
        if ws is None or ws.numel() < need.value:
            ws = torch.empty(max(need.value, 1 << 16), dtype=torch.uint8, device=dev)
            _bufs[key] = ws
        rc = _lib.lib().nvfp4kv_index_topk(q.data_ptr(), q.stride(0), q.stride(1), weights.data_ptr(),
                                           weights.stride(0), pool.data_ptr(), pool.shape[0],
                                           block_tables.data_ptr(), block_tables.stride(0),
                                           seq_lens.contiguous().data_ptr(), B, q.shape[1], int(page_size),
                                           int(max_seq_len), int(topk), out_rows.data_ptr(), out_count.data_ptr(),
                                           ws.data_ptr(), ws.numel(), _err_word(dev).data_ptr(), _stream(dev))
    _lib.check(rc, "nvfp4kv_index_topk")
    return out_rows, out_count


def index_scores_buffer(device=None) -> torch.Tensor | None:
    """The score workspace of the last index_topk on `device` (float32, [B, ceil(max_seq_len /
    128) * 128] row-major), for inspection."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    ws = _bufs.get(("index_ws", dev.index))
    return None if ws is None else ws.view(torch.float32)
