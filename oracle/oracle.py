"""CPU oracle for the NVFP4 paged KV-cache path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline / reference arm may
import this module; the product path (``glm53_flash_dual_dgx_spark_b200``) never does.

Byte-level work (append quantisation, dequantisation, the 656-byte gather) runs in
``nvfp4_oracle.c`` (built by ``oracle/Makefile``); this module wraps it with numpy and
adds the floating-point pieces:

* :func:`quant` -- ``_quant_kernel`` / ``write_nvfp4``
  (reference ``nvfp4-kv/glm53_nvfp4_runtime.py:37-76``), bit-exact semantics.
* :func:`dequant` -- code x block scale, exact in fp32 (``:81-108``).
* :func:`gather_ds656` -- ``_gather_kernel`` (``:87-122``), bit-exact semantics.
* :func:`build_scratch` -- ``build_scratch`` (``:143-182``): the sync-free path for
  ``T <= sync_free_t`` and the ``unique`` path above it.
* :func:`mla_decode` -- ``softmax(bmm1_scale * q K^T) V * bmm2_scale`` over the dequantised
  pool rows, the formula of the reference's ground truth
  (``nvfp4-kv/test_kernel_equiv.py:49-52``), in float64 by default.  The consumer the
  reference feeds (FlashInfer's trtllm-gen MLA decode) is a closed third-party kernel, so
  this part of the oracle is a restatement of the published formula, not a pinned copy.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

NV_BYTES = 288
DS_BYTES = 656
LATENT = 512

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnvfp4_oracle.so")
_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile the C oracle with its Makefile (gcc) and return the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            src = os.path.join(_HERE, "nvfp4_oracle.c")
            if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
                build()
            lib = ctypes.CDLL(_LIB_PATH)
            P = ctypes.c_void_p
            I64 = ctypes.c_int64
            lib.oracle_quant_rows.argtypes = [P, ctypes.c_int, I64, I64, P, I64, P]
            lib.oracle_dequant_rows.argtypes = [P, I64, P, I64, P]
            lib.oracle_gather_ds656.argtypes = [P, I64, P, I64, P]
            lib.oracle_f32_to_e4m3_array.argtypes = [P, I64, P]
            lib.oracle_e4m3_to_f32_array.argtypes = [P, I64, P]
            for fn in ("oracle_quant_rows", "oracle_dequant_rows", "oracle_gather_ds656",
                       "oracle_f32_to_e4m3_array", "oracle_e4m3_to_f32_array"):
                getattr(lib, fn).restype = None
            _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def _as_u16_bits(x) -> tuple[np.ndarray, int]:
    """Accept a torch bf16/fp16 tensor or a numpy uint16/float16 array; return bits + dtype code."""
    try:
        import torch

        if isinstance(x, torch.Tensor):
            if x.dtype == torch.bfloat16:
                return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16), 0
            if x.dtype == torch.float16:
                return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16), 1
            raise TypeError(f"kv_c must be bf16 or fp16, got {x.dtype}")
    except ImportError:  # pragma: no cover - torch is always present in this repo
        pass
    x = np.asarray(x)
    if x.dtype == np.float16:
        return np.ascontiguousarray(x).view(np.uint16), 1
    if x.dtype == np.uint16:  # raw bf16 bits
        return np.ascontiguousarray(x), 0
    raise TypeError(f"kv_c must be bf16 bits (uint16) or float16, got {x.dtype}")


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 bytes, round-to-nearest-even, saturating (cvt.rn.satfinite semantics)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    _load().oracle_f32_to_e4m3_array(_ptr(x), x.size, _ptr(out))
    return out


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.empty(b.shape, dtype=np.float32)
    _load().oracle_e4m3_to_f32_array(_ptr(b), b.size, _ptr(out))
    return out


def quant(kv_c, slot_mapping, pool: np.ndarray) -> np.ndarray:
    """Write NVFP4 rows for ``kv_c`` [T, >=512] at ``slot_mapping`` into ``pool`` (in place).

    ``pool`` is a uint8 array viewable as [rows, 288]; rows whose slot is negative or past
    the pool are skipped, as ``_quant_kernel`` skips ``slot < 0``.
    """
    bits, dtype = _as_u16_bits(kv_c)
    if bits.ndim != 2 or bits.shape[1] < LATENT:
        raise ValueError("kv_c must be [T, >=512]")
    slot = np.ascontiguousarray(np.asarray(slot_mapping).reshape(-1), dtype=np.int64)
    if slot.shape[0] != bits.shape[0]:
        raise ValueError("slot_mapping length must equal T")
    flat = pool.reshape(-1, NV_BYTES)
    if not flat.flags.c_contiguous:
        raise ValueError("pool must be contiguous")
    _load().oracle_quant_rows(_ptr(bits), dtype, bits.shape[0], bits.shape[1], _ptr(flat),
                              flat.shape[0], _ptr(slot))
    return pool


def quant_new(kv_c) -> np.ndarray:
    """Quantise T tokens into a fresh [T, 288] pool (slot t -> row t)."""
    bits, _ = _as_u16_bits(kv_c)
    pool = np.zeros((bits.shape[0], NV_BYTES), dtype=np.uint8)
    quant(kv_c, np.arange(bits.shape[0], dtype=np.int64), pool)
    return pool


def dequant(pool: np.ndarray, rows) -> np.ndarray:
    """Rows of the pool -> float32 [n, 512]; out-of-range rows read as zeros."""
    flat = np.ascontiguousarray(pool.reshape(-1, NV_BYTES))
    rows = np.ascontiguousarray(np.asarray(rows).reshape(-1), dtype=np.int64)
    out = np.empty((rows.shape[0], LATENT), dtype=np.float32)
    _load().oracle_dequant_rows(_ptr(flat), flat.shape[0], _ptr(rows), rows.shape[0], _ptr(out))
    return out


def gather_ds656(pool: np.ndarray, idx, rope=None) -> np.ndarray:
    """``_gather_kernel``: NVFP4 rows at ``idx`` -> [S, 656] fp8_ds_mla rows.  ``rope`` (not in
    the reference, which writes zeros there, runtime:121-122): a side-pool of 64 bf16 bit
    patterns per row (uint16 [rows, 64]) whose clamped row fills the rope bytes [528, 656)."""
    flat = np.ascontiguousarray(pool.reshape(-1, NV_BYTES))
    idx = np.ascontiguousarray(np.asarray(idx).reshape(-1), dtype=np.int32)
    out = np.empty((idx.shape[0], DS_BYTES), dtype=np.uint8)
    _load().oracle_gather_ds656(_ptr(flat), flat.shape[0], _ptr(idx), idx.shape[0], _ptr(out))
    if rope is not None:
        src = np.clip(idx.astype(np.int64), 0, flat.shape[0] - 1)
        out[:, 528:] = np.ascontiguousarray(np.asarray(rope, dtype=np.uint16)[src]).view(np.uint8)
    return out


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def build_scratch(pool: np.ndarray, block_tables, sync_free_t: int = 192):
    """``build_scratch`` (runtime:143-182): returns (scratch [P, 64, 656], tables [T, 1, K]).

    For ``T <= sync_free_t`` every table entry is gathered (no dedup) and the tables are an
    arange; otherwise the entries are deduplicated with ``unique`` and renumbered.
    """
    bt = np.asarray(block_tables)
    T, one, K = bt.shape
    flat = bt.reshape(-1).astype(np.int32)
    if T <= sync_free_t:
        S = T * K
        P = (S + 63) // 64
        rows = gather_ds656(pool, flat)
        scratch = np.zeros((P * 64, DS_BYTES), dtype=np.uint8)
        scratch[:S] = rows
        return scratch.reshape(P, 64, DS_BYTES), np.arange(S, dtype=np.int32).reshape(T, 1, K)
    uniq, inv = np.unique(flat, return_inverse=True)
    S = uniq.shape[0]
    P = (S + 63) // 64
    scratch = np.zeros((P * 64, DS_BYTES), dtype=np.uint8)
    scratch[:S] = gather_ds656(pool, uniq.astype(np.int32))
    return scratch.reshape(P, 64, DS_BYTES), inv.astype(np.int32).reshape(T, 1, K)


def token_rows(block_tables, seq_lens, page_size: int, sparse: bool, pool_rows: int):
    """Per batch entry, (pool rows, token positions) it attends to, invalid entries dropped.

    Dense: token t < seq_lens[b] lives at row ``block_tables[b, t // page] * page + t % page``;
    tokens whose page id is outside the pool are masked.
    Sparse: entries j < seq_lens[b] of ``block_tables[b, 0 or :, j]`` are physical rows;
    negative or out-of-range rows are masked.  The position of entry j is j.
    """
    num_pages = pool_rows // page_size
    bt = np.asarray(block_tables)
    sl = np.asarray(seq_lens).reshape(-1)
    out = []
    for b in range(sl.shape[0]):
        n = int(sl[b])
        t = np.arange(n, dtype=np.int64)
        if sparse:
            idx = bt[b].reshape(-1)[:n].astype(np.int64)
            ok = (idx >= 0) & (idx < pool_rows)
            out.append((idx[ok], t[ok]))
        else:
            pages = bt[b].reshape(-1)[t // page_size].astype(np.int64)
            ok = (pages >= 0) & (pages < num_pages)
            out.append(((pages * page_size + t % page_size)[ok], t[ok]))
    return out


def mla_decode(q, pool: np.ndarray, block_tables, seq_lens, *, sparse: bool,
               page_size: int = 64, bmm1_scale: float = 1.0, bmm2_scale: float = 1.0,
               kv_lora_rank: int = LATENT, dtype=np.float64, return_lse: bool = False, rope=None):
    """Reference attention over the NVFP4 pool.

    q: [B, q_len, H, 576] (any float dtype; the last 64 rope dims multiply the all-zero
    K rope of the 288-byte layout and so contribute nothing, unless ``rope``, a side-pool of 64
    bf16 bit patterns per row (uint16 [rows, 64]), gives the keys a rope part: then
    score = q[:512] . k + q[512:576] . k_rope).  Query token i of a dense
    entry with q_len > 1 sees context tokens ``t < seq_len - (q_len - 1 - i)`` (causal MTP).
    Returns float [B, q_len, H, 512] (and the natural-log LSE [B, q_len, H] if asked).
    """
    try:
        import torch

        if isinstance(q, torch.Tensor):
            q = q.detach().float().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    q = np.asarray(q, dtype=np.float32)
    B, QL, H, D = q.shape
    flat_pool = pool.reshape(-1, NV_BYTES)
    rows = token_rows(block_tables, seq_lens, page_size, sparse, flat_pool.shape[0])
    out = np.zeros((B, QL, H, kv_lora_rank), dtype=dtype)
    lse = np.full((B, QL, H), -np.inf, dtype=dtype)
    sl = np.asarray(seq_lens).reshape(-1)
    for b in range(B):
        r, pos = rows[b]
        kv = dequant(flat_pool, r).astype(dtype)                 # [n, 512]
        kr = bf16_bits_to_f32(np.asarray(rope)[r]).astype(dtype) if rope is not None else None
        for i in range(QL):
            lim = int(sl[b]) if sparse else int(sl[b]) - (QL - 1 - i)
            k = kv[pos < lim]
            if k.shape[0] == 0:
                continue
            s = q[b, i, :, :kv_lora_rank].astype(dtype) @ k.T               # [H, vis]
            if kr is not None:
                s = s + q[b, i, :, kv_lora_rank:kv_lora_rank + 64].astype(dtype) @ kr[pos < lim].T
            s = s * dtype(bmm1_scale)
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - m)
            l = p.sum(axis=1, keepdims=True)
            out[b, i] = (p @ k) / l * dtype(bmm2_scale)
            lse[b, i] = (m + np.log(l))[:, 0]
    if return_lse:
        return out, lse
    return out


# ---------------------------------------------------------------- indexer K-pool
INDEX_DIM = 128
INDEX_ROW = 72


def index_quant(k) -> np.ndarray:
    """128-d indexer keys [T, 128] -> 72-byte NVFP4 rows [T, 72] by the latent rows' rule
    (``_quant_kernel``, runtime:37-65): blocks of 16 are independent, so a key is quantised as
    the first 128 elements of a zero-padded 512-element row and its 64 code bytes and 8 scale
    bytes are kept."""
    try:
        import torch

        if isinstance(k, torch.Tensor):
            k = k.detach().cpu()
            pad = torch.zeros(k.shape[0], LATENT, dtype=k.dtype)
            pad[:, :INDEX_DIM] = k[:, :INDEX_DIM]
            rows = quant_new(pad)
        else:
            raise TypeError
    except (ImportError, TypeError):  # pragma: no cover
        raise TypeError("index_quant takes a bf16/fp16 torch tensor")
    return np.concatenate([rows[:, :64], rows[:, 256:264]], axis=1)


def index_dequant(rows72: np.ndarray) -> np.ndarray:
    """72-byte indexer rows -> float32 [n, 128] (code x scale, exact)."""
    r = np.asarray(rows72, dtype=np.uint8).reshape(-1, INDEX_ROW)
    full = np.zeros((r.shape[0], NV_BYTES), dtype=np.uint8)
    full[:, :64] = r[:, :64]
    full[:, 256:264] = r[:, 64:72]
    return dequant(full, np.arange(r.shape[0]))[:, :INDEX_DIM]


def index_scores(q, weights, pool72: np.ndarray, tables, seq_lens, page_size: int = 64):
    """Per entry b, float64 scores of its visible positions s < seq_lens[b]:
    sum_h w[b, h] * max(q[b, h] . k[s], 0) (DeepSeek-V3.2's indexer rule), -inf where the
    position's page is outside the pool."""
    try:
        import torch

        if isinstance(q, torch.Tensor):
            q = q.detach().float().cpu().numpy()
        if isinstance(weights, torch.Tensor):
            weights = weights.detach().float().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    flat = np.asarray(pool72, dtype=np.uint8).reshape(-1, INDEX_ROW)
    keys = index_dequant(flat).astype(np.float64)
    num_pages = flat.shape[0] // page_size
    out = []
    for b in range(len(seq_lens)):
        n = int(seq_lens[b])
        pos = np.arange(n)
        pages = np.asarray(tables[b])[pos // page_size].astype(np.int64)
        ok = (pages >= 0) & (pages < num_pages)
        rows = np.where(ok, pages * page_size + pos % page_size, 0)
        dots = keys[rows] @ np.asarray(q[b], dtype=np.float64).T          # [n, H]
        s = np.maximum(dots, 0.0) @ np.asarray(weights[b], dtype=np.float64)
        out.append(np.where(ok, s, -np.inf))
    return out


def index_select(scores_b: np.ndarray, topk: int) -> np.ndarray:
    """Positions of the topk largest scores, ascending; ties at the threshold to the lowest
    positions (the selection rule of nvfp4kv_index_topk)."""
    n = scores_b.shape[0]
    if n <= topk:
        return np.arange(n)
    order = np.lexsort((np.arange(n), -scores_b))        # score descending, then position
    return np.sort(order[:topk])
