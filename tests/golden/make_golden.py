"""Generate the golden fixtures in this directory from the reference implementation.

Run in a container that has the reference checkout (``--reference`` points at the
directory holding ``nvfp4-kv/glm53_nvfp4_runtime.py``):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --reference <path-to-reference>

The reference's Triton kernels (``_quant_kernel``, ``_gather_kernel``) and its
``build_scratch`` run unmodified on the CPU through the Triton interpreter, which executes
them with numpy's IEEE fp32 arithmetic.  Three interpreter behaviours are not IEEE (nor
what the kernels compile to on a GPU) and are corrected by patching the *interpreter*
(never the reference):

1. ``_convert_float`` (fp32 <-> fp8e4nv) rounds ties away from zero, drops mantissa carries
   and does not saturate.  GPU code uses ``cvt.rn.satfinite.e4m3x2.f32``: round to nearest
   even, saturate to +-448, NaN -> 0x7f.  The patch uses torch's float8_e4m3fn cast (an
   independent RNE implementation) after a clamp to +-448.
2. ``_convert_float`` (bf16 -> fp32) mangles subnormal bf16 values (6.4e-40 becomes
   8.8e-39); the patch widens exactly.
3. ``create_maxnumf`` maps to ``np.maximum`` (NaN-propagating); ``tl.maximum`` lowers to
   ``maxnum`` on the GPU, which returns the non-NaN operand.  The patch uses ``np.fmax``.

The unpatched interpreter output is stored too (``*_raw``) so the size of divergence (1)
stays on record.  Outputs: quant_golden.npz, gather_golden.npz, scratch_golden.npz.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ["GLM53_NVFP4_KV"] = "1"

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def quant_inputs() -> torch.Tensor:
    """96 tokens: 64 rows ~N(0,1) (seed 0, the distribution of config 1) + edge cases."""
    g = torch.Generator().manual_seed(0)
    rows = [torch.randn(64, 512, generator=g)]
    e = []
    e.append(torch.zeros(512))                                   # 64: all zero -> 0x77, scale 0
    r = torch.randn(512, generator=g); r[:16] = 0; e.append(r)  # 65: one zero block
    e.append(torch.randn(512, generator=g) * 1e-6)               # 66: scale underflows to 0
    e.append(torch.randn(512, generator=g) * 1e4)                # 67: large blocks
    r = torch.randn(512, generator=g)
    r[torch.randperm(512, generator=g)[:6]] *= 20.0              # 68: 1% outliers x20
    e.append(r)
    # 69: exact threshold ties.  Block max 6*s with s = 0.5 (exact e4m3) so the scale is s
    # and elements sit exactly on t*s for every ladder threshold t.
    r = torch.zeros(512)
    s = 0.5
    th = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0])
    for blk in range(32):
        vals = torch.cat([th * s, -th * s]) * (1.0 if blk % 2 == 0 else 1.0)
        r[16 * blk:16 * blk + 16] = vals
    e.append(r)
    r = torch.randn(512, generator=g) * 1e-3; r[::3] = -0.0; e.append(r)   # 70: signed zeros
    r = torch.randn(512, generator=g); r[5] = float("inf"); r[300] = float("-inf"); e.append(r)  # 71
    r = torch.randn(512, generator=g); r[40] = float("nan"); e.append(r)   # 72: one NaN element
    r = torch.randn(512, generator=g); r[64:80] = float("nan"); e.append(r)  # 73: all-NaN block
    # 74: block maxima m*2^k with m/3 an odd 5-bit integer: amax/6 is an exact e4m3 tie.
    r = torch.randn(512, generator=g) * 0.1
    ms = [51, 57, 63, 69, 75, 81, 87, 93]
    for blk in range(32):
        r[16 * blk] = ms[blk % 8] * 2.0 ** ((blk // 8) - 4)
    e.append(r)
    r = torch.randn(512, generator=g) * 1e-39; e.append(r)      # 75: bf16 subnormal inputs
    for k in range(20):                                          # 76-95: scales 2^-12 .. 2^7
        e.append(torch.randn(512, generator=g) * 2.0 ** (k - 12))
    rows.append(torch.stack(e))
    return torch.cat(rows).to(torch.bfloat16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "nvfp4-kv"))

    import triton.language as tl
    import triton.runtime.interpreter as interp

    import glm53_nvfp4_runtime as rt  # the reference runtime, unmodified

    orig_convert = interp._convert_float
    orig_maxnumf = interp.InterpreterBuilder.create_maxnumf

    def faithful_convert(inp, in_dt, out_dt, rounding_mode):
        if in_dt == tl.float32 and out_dt == tl.float8e4nv:
            x = torch.from_numpy(np.ascontiguousarray(inp).view(np.float32).copy())
            y = x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).clone()
            y[torch.isnan(x)] = 0x7F
            return y.numpy().reshape(inp.shape)
        if in_dt == tl.bfloat16 and out_dt == tl.float32:
            b = torch.from_numpy(np.ascontiguousarray(inp).view(np.int16).copy())
            f = b.view(torch.bfloat16).float()
            return f.numpy().view(np.uint32).reshape(inp.shape)
        if in_dt == tl.float8e4nv and out_dt == tl.float32:
            b = torch.from_numpy(np.ascontiguousarray(inp).view(np.uint8).copy())
            f = b.view(torch.float8_e4m3fn).float()
            return f.numpy().view(np.uint32).reshape(inp.shape)
        return orig_convert(inp, in_dt, out_dt, rounding_mode)

    def set_faithful(on: bool) -> None:
        interp._convert_float = faithful_convert if on else orig_convert
        interp.InterpreterBuilder.create_maxnumf = (
            (lambda self, lhs, rhs: self.binary_op(lhs, rhs, np.fmax)) if on else orig_maxnumf)

    # ------------------------------------------------------------------ append
    kv = quant_inputs()
    T = kv.shape[0]
    g = torch.Generator().manual_seed(1)
    pool_rows = 128
    slot = torch.randperm(pool_rows, generator=g)[:T].to(torch.int64)
    slot[torch.tensor([3, 17, 90])] = -1
    pool_init = torch.randint(0, 256, (pool_rows, 288), dtype=torch.uint8, generator=g)
    outs = {}
    for name, on in (("pool_ref", True), ("pool_ref_raw", False)):
        set_faithful(on)
        pool = pool_init.clone()
        rt.write_nvfp4(kv, pool.view(pool_rows // 64, 64, 288), slot)
        outs[name] = pool.numpy().copy()
    # fp16 input with a row stride wider than 512 (a [T, 576] buffer, latent in :512)
    g16 = torch.Generator().manual_seed(2)
    wide = (torch.randn(16, 576, generator=g16) * 3).to(torch.float16)
    set_faithful(True)
    pool16 = torch.zeros(16, 288, dtype=torch.uint8)
    rt.write_nvfp4(wide[:, :512], pool16, torch.arange(16))
    np.savez_compressed(
        os.path.join(HERE, "quant_golden.npz"),
        kv_c_bf16_bits=_bf16_bits(kv), slot_mapping=slot.numpy(), pool_init=pool_init.numpy(),
        pool_ref=outs["pool_ref"], pool_ref_raw=outs["pool_ref_raw"],
        wide_f16=wide.numpy(), pool16_ref=pool16.numpy())

    # ------------------------------------------------------------------ gather
    gg = torch.Generator().manual_seed(0)
    R = 512
    pool = torch.randint(0, 256, (R, 288), dtype=torch.uint8, generator=gg)   # raw bytes, as test_syncfree.py
    qrows = torch.randn(128, 512, generator=gg).to(torch.bfloat16)
    qpool = torch.zeros(128, 288, dtype=torch.uint8)
    set_faithful(True)
    rt.write_nvfp4(qrows, qpool, torch.arange(128))
    pool[R - 128:] = qpool                                                      # realistic rows too
    S = 300
    idx = torch.randint(0, R, (S,), dtype=torch.int32, generator=gg)
    idx[torch.randperm(S, generator=gg)[:30]] = -1                             # 10% padding
    idx[7] = R + 5                                                              # out of range -> clamp
    idx[8] = -7
    res = {}
    for name, on in (("out_ref", True), ("out_ref_raw", False)):
        set_faithful(on)
        out = torch.zeros(S, 656, dtype=torch.uint8)
        rt._gather(pool, idx, out)
        res[name] = out.numpy().copy()
    np.savez_compressed(os.path.join(HERE, "gather_golden.npz"), pool=pool.numpy(), idx=idx.numpy(),
                        out_ref=res["out_ref"], out_ref_raw=res["out_ref_raw"])

    # ------------------------------------------------------------------ build_scratch
    set_faithful(True)
    gs = torch.Generator().manual_seed(3)
    small_pool = pool[:200].clone()
    cases = {}
    for T_, K_ in ((3, 64), (5, 64)):
        bt = torch.randint(0, 200, (T_, 1, K_), dtype=torch.int32, generator=gs)
        bt[:, :, : K_ // 4] = bt[:1, :, : K_ // 4]                             # cross-token duplicates
        bt[torch.rand(T_, 1, K_, generator=gs) < 0.1] = -1
        rt._bufs.clear()
        sa, ta = rt.build_scratch(small_pool, bt)
        saved = rt._SYNC_FREE_T
        rt._SYNC_FREE_T = 0
        try:
            sb, tb = rt.build_scratch(small_pool, bt)
        finally:
            rt._SYNC_FREE_T = saved
        cases[f"bt_{T_}"] = bt.numpy()
        cases[f"sync_scratch_{T_}"] = sa.numpy().copy()
        cases[f"sync_tables_{T_}"] = ta.numpy().copy()
        cases[f"uniq_scratch_{T_}"] = sb.numpy().copy()
        cases[f"uniq_tables_{T_}"] = tb.numpy().copy()
    np.savez_compressed(os.path.join(HERE, "scratch_golden.npz"), pool=small_pool.numpy(), **cases)
    set_faithful(False)
    print("wrote quant_golden.npz gather_golden.npz scratch_golden.npz")


if __name__ == "__main__":
    main()
