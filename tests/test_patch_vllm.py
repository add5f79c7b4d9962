"""CPU: the vLLM 0.22 seam patcher (glm53_flash_dual_dgx_spark_b200/patch_vllm.py).

The patcher runs on copies of the installed vLLM 0.22 files (the installed tree is never
written).  Checked: every seam applies and the files still parse; a second run changes
nothing; an anchor that drifted aborts with nothing written (fail closed); --check writes
nothing; and the patched functions behave: with the NVFP4 path enabled the fp8_ds_mla page
is 288 B, the pool shape [blocks, block_size, 288] and the write goes to write_nvfp4, and
disabled they are the stock behaviour.  The patched functions are pulled out of the copies
with ``ast`` and run against fake ``vllm.glm53_nvfp4_runtime`` / ``vllm._custom_ops``
modules, so nothing of vLLM itself is imported.
"""
import ast
import importlib.util
import os
import shutil
import sys
import textwrap
import types

import pytest
import torch

from glm53_flash_dual_dgx_spark_b200 import patch_vllm as PV


def _vllm_root():
    spec = importlib.util.find_spec("vllm")
    if spec is None or not spec.submodule_search_locations:
        pytest.skip("vllm is not installed")
    return list(spec.submodule_search_locations)[0]


@pytest.fixture
def tree(tmp_path):
    src = _vllm_root()
    root = tmp_path / "vllm"
    for rel in sorted({s.path for s in PV.SEAMS}):
        os.makedirs(root / os.path.dirname(rel), exist_ok=True)
        shutil.copy(os.path.join(src, rel), root / rel)
    return str(root)


def _read_all(root):
    out = {}
    for dirpath, _, files in os.walk(root):
        for f in files:
            p = os.path.join(dirpath, f)
            with open(p, "rb") as fh:
                out[os.path.relpath(p, root)] = fh.read()
    return out


def test_every_seam_applies_and_the_files_parse(tree):
    log = PV.apply(tree)
    assert sum(line.endswith(": patched") for line in log) == len(PV.SEAMS)
    for rel in {s.path for s in PV.SEAMS}:
        text = open(os.path.join(tree, rel)).read()
        ast.parse(text)
        assert PV.MARK in text
    shim = open(os.path.join(tree, PV.RUNTIME_MODULE)).read()
    ast.parse(shim)
    assert "glm53_flash_dual_dgx_spark_b200.glm53_nvfp4_runtime" in shim


def test_second_run_changes_nothing(tree):
    PV.apply(tree)
    before = _read_all(tree)
    log = PV.apply(tree)
    assert not any(line.endswith(": patched") for line in log)
    assert sum("already patched" in line for line in log) == len(PV.SEAMS)
    assert _read_all(tree) == before


def test_anchor_drift_fails_closed_with_nothing_written(tree, capsys):
    rel = "v1/attention/backends/mla/flashinfer_mla_sparse.py"
    p = os.path.join(tree, rel)
    text = open(p).read().replace("trtllm_batch_decode_with_kv_cache_mla(\n            query=q.unsqueeze(1),",
                                  "trtllm_batch_decode_with_kv_cache_mla(\n            query=q,", 1)
    open(p, "w").write(text)
    before = _read_all(tree)
    with pytest.raises(PV.AnchorDrift, match="read path"):
        PV.apply(tree)
    assert _read_all(tree) == before                    # not even the other files' seams
    assert PV.main(["--vllm-root", tree]) == 1
    assert "ANCHOR DRIFT" in capsys.readouterr().err


def test_duplicate_anchor_is_drift(tree):
    p = os.path.join(tree, "v1/kv_cache_interface.py")
    text = open(p).read()
    anchor = PV.SEAMS[0].old
    open(p, "w").write(text + "\n" + textwrap.indent(anchor, ""))
    with pytest.raises(PV.AnchorDrift, match="2 times"):
        PV.apply(tree)


def test_check_mode_writes_nothing(tree):
    before = _read_all(tree)
    assert PV.main(["--vllm-root", tree, "--check"]) == 0
    assert _read_all(tree) == before


# ---------------------------------------------------------------- behaviour of patched code
def _function(path, name, cls=None):
    text = open(path).read()
    mod = ast.parse(text)
    scope = mod.body
    if cls:
        scope = next(n for n in mod.body if isinstance(n, ast.ClassDef) and n.name == cls).body
    node = next(n for n in scope if isinstance(n, ast.FunctionDef) and n.name == name)
    # the segment starts at "def" (decorators such as @property / @staticmethod are left out)
    return textwrap.dedent(ast.get_source_segment(text, node, padded=True))


@pytest.fixture
def fake_vllm(monkeypatch):
    calls = []
    rt = types.ModuleType("vllm.glm53_nvfp4_runtime")
    rt.NV_BYTES, rt.DS_BYTES = 288, 656
    rt.on = True
    rt.enabled = lambda: rt.on
    rt.write_nvfp4 = lambda kv_c, kv_cache, slot: calls.append(("write_nvfp4", slot))
    ops = types.ModuleType("vllm._custom_ops")
    ops.concat_and_cache_mla = lambda *a, **k: calls.append(("concat_and_cache_mla", k["kv_cache_dtype"]))
    pkg = types.ModuleType("vllm")
    pkg.glm53_nvfp4_runtime, pkg._custom_ops = rt, ops
    monkeypatch.setitem(sys.modules, "vllm", pkg)
    monkeypatch.setitem(sys.modules, "vllm.glm53_nvfp4_runtime", rt)
    monkeypatch.setitem(sys.modules, "vllm._custom_ops", ops)
    return rt, calls


def _load(src, **glb):
    ns = dict(glb, torch=torch)
    exec(compile(src, "<patched>", "exec"), ns)
    return ns


def test_patched_pool_bytes_and_shape(tree, fake_vllm):
    rt, _ = fake_vllm
    PV.apply(tree)
    f = _load(_function(os.path.join(tree, "v1/kv_cache_interface.py"), "real_page_size_bytes",
                        "MLAAttentionSpec"))["real_page_size_bytes"]
    spec = types.SimpleNamespace(cache_dtype_str="fp8_ds_mla", model_version="deepseek_v32", block_size=64,
                                 storage_block_size=64, num_kv_heads=1, head_size=576,
                                 dtype=torch.uint8, compress_ratio=1)
    assert f(spec) == 64 * 288
    rt.on = False
    assert f(spec) == 64 * 656
    g = _load(_function(os.path.join(tree, "v1/attention/backends/mla/flashinfer_mla_sparse.py"),
                        "get_kv_cache_shape", "FlashInferMLASparseBackend"))["get_kv_cache_shape"]
    assert g(100, 64, 1, 576, "auto") == (100, 64, 576)
    assert g(100, 64, 1, 576, "fp8_ds_mla") == (100, 64, 656)
    rt.on = True
    assert g(100, 64, 1, 576, "fp8_ds_mla") == (100, 64, 288)
    assert g(100, 64, 1, 576, "bfloat16") == (100, 64, 576)


def test_patched_write_path_dispatch(tree, fake_vllm):
    rt, calls = fake_vllm
    PV.apply(tree)
    f = _load(_function(os.path.join(tree, "v1/attention/backend.py"), "do_kv_cache_update",
                        "SparseMLAAttentionImpl"))["do_kv_cache_update"]
    kv = torch.zeros(2, 64, 288, dtype=torch.uint8)
    slot = torch.arange(4).view(2, 2)
    args = (None, torch.zeros(4, 512), torch.zeros(4, 1, 64), kv, slot)
    f(*args, "fp8_ds_mla", torch.tensor(1.0))
    assert calls[-1][0] == "write_nvfp4" and calls[-1][1].shape == (4,)      # slot_mapping flattened
    f(*args, "auto", torch.tensor(1.0))
    assert calls[-1] == ("concat_and_cache_mla", "auto")
    rt.on = False
    f(*args, "fp8_ds_mla", torch.tensor(1.0))
    assert calls[-1] == ("concat_and_cache_mla", "fp8_ds_mla")
    # the dense-MLA do_kv_cache_update (same body in 0.22) is untouched
    dense = _function(os.path.join(tree, "v1/attention/backend.py"), "do_kv_cache_update", "MLAAttentionImpl")
    assert PV.MARK not in dense
