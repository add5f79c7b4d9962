"""GPU: nvfp4_append (C ABI, via the drop-in write_nvfp4) is bit-exact with the reference
goldens and with the oracle, including configuration 1 of the benchmark set."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    rt.device_errors()
    return rt


def _bf16_from_bits(bits):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


def test_append_matches_reference_golden(rt):
    d = np.load(os.path.join(GOLDEN, "quant_golden.npz"))
    kv = _bf16_from_bits(d["kv_c_bf16_bits"]).cuda()
    pool = torch.from_numpy(d["pool_init"].copy()).cuda()
    slot = torch.from_numpy(d["slot_mapping"]).cuda()
    rt.write_nvfp4(kv, pool.view(2, 64, 288), slot)
    got = pool.cpu().numpy()
    bad = np.argwhere(got != d["pool_ref"])
    assert bad.size == 0, f"{len(bad)} bytes differ, first {bad[:8].tolist()}"
    assert rt.device_errors() == 0


def test_append_fp16_strided_matches_reference_golden(rt):
    d = np.load(os.path.join(GOLDEN, "quant_golden.npz"))
    wide = torch.from_numpy(d["wide_f16"]).cuda()
    pool = torch.zeros(16, 288, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(wide[:, :512], pool, torch.arange(16, device="cuda"))
    assert np.array_equal(pool.cpu().numpy(), d["pool16_ref"])


def test_append_config1_bit_exact_and_round_trip(rt):
    """Config 1: 4 seqs x 4096 tokens, latent N(0,1) bf16 (seed 0), rope N(0,1) ignored,
    page 64, slots on shuffled pages; codes + scales bit-exact, round trip rel ~0.1."""
    torch.manual_seed(0)
    T = 4 * 4096
    latent = torch.randn(T, 512).to(torch.bfloat16)
    rope = torch.randn(T, 64).to(torch.bfloat16)            # dropped, as the reference does
    kv_c = torch.cat([latent, rope], dim=1)                  # [T, 576]: latent is a strided view
    pages = torch.randperm(T // 64)
    slot = (pages.repeat_interleave(64) * 64 + torch.arange(64).repeat(T // 64)).to(torch.int64)
    pool = torch.zeros(T // 64, 64, 288, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(kv_c.cuda()[:, :512], pool, slot.cuda())
    ref = np.zeros((T, 288), np.uint8)
    O.quant(latent, slot.numpy(), ref)
    assert np.array_equal(pool.view(-1, 288).cpu().numpy(), ref)
    y = O.dequant(ref, slot.numpy())
    rel = np.linalg.norm(y - latent.float().numpy()) / np.linalg.norm(latent.float().numpy())
    assert 0.08 < rel < 0.13


@pytest.mark.parametrize("scale", [1e-3, 1.0, 37.0, 3e4])
def test_append_int32_slots_and_value_ranges(rt, scale):
    g = torch.Generator().manual_seed(5)
    T = 777
    x = (torch.randn(T, 512, generator=g) * scale)
    x[torch.rand(T, 512, generator=g) < 0.01] *= 20.0        # config 5's outliers
    x = x.to(torch.bfloat16)
    slot = torch.randperm(1024, generator=g)[:T].to(torch.int32)
    slot[::50] = -1
    pool = torch.zeros(1024, 288, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(x.cuda(), pool, slot.cuda())
    ref = np.zeros((1024, 288), np.uint8)
    O.quant(x, slot.numpy().astype(np.int64), ref)
    assert np.array_equal(pool.cpu().numpy(), ref)


def test_append_out_of_range_slot_is_skipped_and_flagged(rt):
    x = torch.randn(4, 512, device="cuda").to(torch.bfloat16)
    pool = torch.full((8, 288), 0xAB, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(x, pool, torch.tensor([0, 8, -1, 100], device="cuda"))
    p = pool.cpu().numpy()
    assert (p[1:] == 0xAB).all() and not (p[0] == 0xAB).all()
    assert rt.device_errors() & 2


def test_append_empty_is_noop(rt):
    pool = torch.zeros(4, 288, dtype=torch.uint8, device="cuda")
    rt.write_nvfp4(torch.empty(0, 512, dtype=torch.bfloat16, device="cuda"), pool,
                   torch.empty(0, dtype=torch.int64, device="cuda"))
    assert int(pool.sum()) == 0


def test_append_rejects_cpu_tensors(rt):
    with pytest.raises(ValueError, match="CUDA"):
        rt.write_nvfp4(torch.zeros(2, 512, dtype=torch.bfloat16), torch.zeros(2, 288, dtype=torch.uint8),
                       torch.arange(2))
