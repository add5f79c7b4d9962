"""Append edge cases: bit-exact against the oracle on inputs placed at the quantiser's
decision points.

`_quant_kernel` (nvfp4-kv/glm53_nvfp4_runtime.py:51-64) walks the ladder |x/s| < 0.25,
0.75, 1.25, 1.75, 2.5, 3.5, 5 with ties going up.  The rows built here put elements exactly
on every threshold t*s for e4m3 scales drawn over the whole positive range, on their bf16/fp16 neighbours, on the
e2m1 grid points, and add -0.0, NaN (single, leading and whole-block), +-inf, blocks whose
scale byte is 0, saturated scales and subnormal inputs, in bf16 and fp16, through the
vectorised and the strided load paths.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

THRESH = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
E4M3 = np.array([(m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
                 for c in range(1, 127) for e, m in [(c >> 3, c & 7)]], np.float32)


def _neighbour(v, dtype, step):
    """The next representable value of `dtype` above (step 1) or below (step -1) |v|, signed as v."""
    t = torch.tensor(np.abs(v), dtype=torch.float32).to(dtype)
    bits = t.view(torch.int16) + step
    return float(np.sign(v)) * bits.view(dtype).float().numpy()


def edge_rows(dtype, n_tie=192, seed=2026):
    """[n_tie + 8, 512] tensor of `dtype`; the first n_tie tokens hold ties (see module doc)."""
    rng = np.random.default_rng(seed)
    rows = []
    for _ in range(n_tie):
        row = np.empty(512, np.float32)
        for blk in range(32):
            s = float(E4M3[rng.integers(len(E4M3))])
            v = np.empty(16, np.float32)
            v[0] = 6.0 * s * rng.choice([-1.0, 1.0])                  # the block amax: scale = s
            for i in range(1, 16):
                kind = rng.integers(5)
                sign = rng.choice([-1.0, 1.0])
                if kind == 0:
                    v[i] = sign * THRESH[rng.integers(7)] * s          # exact tie
                elif kind == 1:
                    v[i] = _neighbour(sign * THRESH[rng.integers(7)] * s, dtype, 1)
                elif kind == 2:
                    v[i] = _neighbour(sign * THRESH[rng.integers(7)] * s, dtype, -1)
                elif kind == 3:
                    v[i] = sign * GRID[rng.integers(8)] * s
                else:
                    v[i] = rng.uniform(-6.0, 6.0) * s
            v[rng.integers(1, 16)] = -0.0 if rng.random() < 0.5 else v[rng.integers(1, 16)]
            row[16 * blk:16 * blk + 16] = v[rng.permutation(16)]
        rows.append(row)
    big = 3000.0 if dtype == torch.bfloat16 else 60000.0
    special = np.array([rng.standard_normal(512) for _ in range(8)], np.float32)
    special[0, :] = 0.0
    special[0, 1::3] = -0.0                                           # all-zero row: scale 0
    special[1, 40] = np.nan                                           # one NaN in block 2
    special[2, 64:80] = np.nan                                        # a whole NaN block
    special[2, 96] = np.nan                                           # leading NaN of block 6
    special[3, 5], special[3, 300], special[3, 301] = np.inf, -np.inf, np.inf
    special[4, :] = rng.uniform(-0.004, 0.004, 512)                   # every scale byte 0
    special[4, 256:272] = rng.standard_normal(16)                     # ... but one block
    special[5, :16] = rng.uniform(-big, big, 16)
    special[5, 0] = big                                               # saturated scale (448)
    special[6, :] = rng.standard_normal(512) * 2688.0 / 4.0
    special[6, ::16] = 2688.0                                         # scale 448 in every block
    special[7, :] = rng.standard_normal(512)
    x = torch.from_numpy(np.concatenate([np.array(rows), special])).to(dtype)
    bits = x.view(torch.int16)
    if dtype == torch.bfloat16:
        sub = torch.tensor([0x0001, -0x7FFF, 0x007F, -0x7F81, 0x0040], dtype=torch.int16)  # +-subnormals
        bits[-2, 1:6] = sub
    else:
        sub = torch.tensor([0x0001, -0x7FFF, 0x03FF, -0x7C01, 0x0200], dtype=torch.int16)
        bits[-1, 17:22] = sub                                          # fp16 subnormals, scale ~ N(0,1)
    return x


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_oracle_ties_round_up(dtype):
    """The oracle itself (CPU): an element exactly on t*s gets the code above the threshold,
    its lower neighbour the code below, -0.0 gets code 0, a NaN element code 7."""
    s = 0.375                                  # e4m3 0x2c
    block = np.zeros(16, np.float32)
    block[0] = 6.0 * s
    block[1:8] = THRESH * s
    block[8:15] = [_neighbour(t * s, dtype, -1) for t in THRESH]
    block[15] = -0.0
    x = torch.from_numpy(np.tile(block, 32)[None]).to(dtype)
    row = O.quant_new(x)[0]
    codes = np.stack([row[:8] & 15, row[:8] >> 4], 1).reshape(-1)
    assert codes[0] == 7
    assert list(codes[1:8]) == [1, 2, 3, 4, 5, 6, 7]
    assert list(codes[8:15]) == [0, 1, 2, 3, 4, 5, 6]
    assert codes[15] == 0
    x2 = x.clone()
    x2[0, 2] = float("nan")
    row2 = O.quant_new(x2)[0]
    assert (row2[1] & 15) == 7 and row2[256] == row[256]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("stride", [512, 515])
def test_append_edges_bit_exact(dtype, stride):
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    x = edge_rows(dtype)
    T = x.shape[0]
    wide = torch.zeros(T, stride, dtype=dtype)
    wide[:, :512] = x
    slot = torch.randperm(T + 16, generator=torch.Generator().manual_seed(3))[:T].to(torch.int64)
    pool = torch.zeros(T + 16, 288, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(wide.cuda()[:, :512], pool, slot.cuda())
    ref = np.zeros((T + 16, 288), np.uint8)
    O.quant(x, slot.numpy(), ref)
    got = pool.cpu().numpy()
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} bytes differ, first (row, byte) {bad[:8].tolist()}"
    assert rt.device_errors() == 0
