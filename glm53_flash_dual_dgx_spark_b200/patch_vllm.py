"""Boot-time installer of the NVFP4 KV-cache path into vLLM 0.22 (fails closed on anchor drift).

    python -m glm53_flash_dual_dgx_spark_b200.patch_vllm [--vllm-root DIR] [--check]

Mirrors the reference's patcher (nvfp4-kv/patch_nvfp4_kv.py): the same marker, the same
seams, inert unless GLM53_NVFP4_KV=1, and the same failure behaviour: a seam whose anchor is
not found exactly once aborts with a non-zero exit.  Here every anchor of every file is
checked before any file is written, so a drifted tree is left untouched.  The reference
targets its vLLM fork; this file targets the vLLM 0.22 tree, where the seams are:

  pool bytes   v1/kv_cache_interface.py, real_page_size_bytes: the fp8_ds_mla (V3.2 MLA)
               page is 288 B per token instead of 656 (reference seam 1);
  backend      v1/attention/backends/mla/flashinfer_mla_sparse.py: FlashInfer sparse MLA
               accepts the fp8_ds_mla cache dtype, whose pool shape is
               [blocks, block_size, 288] (reference seam 2), and takes a bf16 query;
  write        v1/attention/backend.py, SparseMLAAttentionImpl.do_kv_cache_update: the
               latent is quantised into the 288-byte rows by write_nvfp4 instead of
               concat_and_cache_mla (reference seam 3; 0.22 has a second, dense-MLA
               do_kv_cache_update with the same body, so the anchor includes the line before);
  read         the same backend's forward_mqa: the fused mla_decode reads the pool directly
               instead of trtllm_batch_decode_with_kv_cache_mla over a gathered scratch
               (reference seam 4 did build_scratch + trtllm).

The reference's fifth patch (a unified-memory free-memory check of its GB10 host) is not on
the KV path and is not carried over.  The runtime is installed as vllm/glm53_nvfp4_runtime.py,
a module that re-exports glm53_flash_dual_dgx_spark_b200.glm53_nvfp4_runtime (the package
must be importable in vLLM's Python environment).
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
from dataclasses import dataclass

MARK = "# [glm53-nvfp4-kv]"
RUNTIME_MODULE = "glm53_nvfp4_runtime.py"


@dataclass(frozen=True)
class Seam:
    path: str      # relative to the vllm package directory
    label: str
    old: str
    new: str


SEAMS = [
    Seam("v1/kv_cache_interface.py", "pool bytes",
         """            # V3.2 main MLA: 656-byte custom layout (kv_lora_rank=512 +
            # qk_rope_head_dim=64, head_size=576). See flashmla_sparse.py.
            return self.block_size * 656""",
         f"""            # V3.2 main MLA: 656-byte custom layout (kv_lora_rank=512 +
            # qk_rope_head_dim=64, head_size=576). See flashmla_sparse.py.
            from vllm import glm53_nvfp4_runtime as _nvR  {MARK}
            if _nvR.enabled():
                return self.block_size * _nvR.NV_BYTES  {MARK} NVFP4 rows
            return self.block_size * 656"""),
    Seam("v1/attention/backends/mla/flashinfer_mla_sparse.py", "cache dtypes",
         """        "fp8",
        "fp8_e4m3",
    ]""",
         f"""        "fp8",
        "fp8_e4m3",
    ]
    from vllm import glm53_nvfp4_runtime as _nvR  {MARK}
    if _nvR.enabled():
        supported_kv_cache_dtypes = [*supported_kv_cache_dtypes, "fp8_ds_mla"]  {MARK}
    del _nvR"""),
    Seam("v1/attention/backends/mla/flashinfer_mla_sparse.py", "cache shape",
         """        cache_dtype_str: str = "auto",
    ) -> tuple[int, ...]:
        return (num_blocks, block_size, head_size)""",
         f"""        cache_dtype_str: str = "auto",
    ) -> tuple[int, ...]:
        if cache_dtype_str == "fp8_ds_mla":  {MARK}
            from vllm import glm53_nvfp4_runtime as _nvR
            return (num_blocks, block_size, _nvR.NV_BYTES if _nvR.enabled() else _nvR.DS_BYTES)
        return (num_blocks, block_size, head_size)"""),
    Seam("v1/attention/backends/mla/flashinfer_mla_sparse.py", "bf16 query",
         """        self.supports_quant_query_input = True""",
         f"""        self.supports_quant_query_input = True
        from vllm import glm53_nvfp4_runtime as _nvR  {MARK}
        if _nvR.enabled() and kv_cache_dtype == "fp8_ds_mla":
            self.supports_quant_query_input = False  {MARK} the NVFP4 decode takes bf16 q"""),
    Seam("v1/attention/backend.py", "write path",
         '''        """MQA-style decode forward pass."""
        raise NotImplementedError

    def do_kv_cache_update(
        self,
        kv_c_normed: torch.Tensor,
        k_pe: torch.Tensor,
        kv_cache: torch.Tensor,
        slot_mapping: torch.Tensor,
        kv_cache_dtype: str,
        k_scale: torch.Tensor,
    ) -> None:
        if kv_cache.numel() == 0:
            return
        from vllm import _custom_ops as ops
''',
         f'''        """MQA-style decode forward pass."""
        raise NotImplementedError

    def do_kv_cache_update(
        self,
        kv_c_normed: torch.Tensor,
        k_pe: torch.Tensor,
        kv_cache: torch.Tensor,
        slot_mapping: torch.Tensor,
        kv_cache_dtype: str,
        k_scale: torch.Tensor,
    ) -> None:
        if kv_cache.numel() == 0:
            return
        from vllm import _custom_ops as ops
        from vllm import glm53_nvfp4_runtime as _nvR  {MARK}
        if _nvR.enabled() and kv_cache_dtype == "fp8_ds_mla":
            # the 288-byte row holds the 512-d latent (k_pe of this NoPE model is zero)
            _nvR.write_nvfp4(kv_c_normed, kv_cache, slot_mapping.flatten())
            return
'''),
    Seam("v1/attention/backends/mla/flashinfer_mla_sparse.py", "read path",
         """        o = trtllm_batch_decode_with_kv_cache_mla(
            query=q.unsqueeze(1),
            kv_cache=kv_c_and_k_pe_cache.unsqueeze(1),""",
         f"""        from vllm import glm53_nvfp4_runtime as _nvR  {MARK}
        _decode = trtllm_batch_decode_with_kv_cache_mla
        if _nvR.enabled() and self.kv_cache_dtype == "fp8_ds_mla":
            # fused gather + dequantise + attention straight from the 288-byte pool
            _decode = _nvR.mla_decode
        o = _decode(
            query=q.unsqueeze(1),
            kv_cache=kv_c_and_k_pe_cache.unsqueeze(1),"""),
]

RUNTIME_SHIM = f'''{MARK} installed by glm53_flash_dual_dgx_spark_b200.patch_vllm
"""The NVFP4 paged KV-cache runtime under the module name vLLM's patched seams import."""
from glm53_flash_dual_dgx_spark_b200.glm53_nvfp4_runtime import *  # noqa: F401,F403
from glm53_flash_dual_dgx_spark_b200.glm53_nvfp4_runtime import (  # noqa: F401
    DS_BYTES, NV_BYTES, _SYNC_FREE_T, _bufs, _gather, build_scratch, enabled, mla_decode,
    mla_decode_lse, write_nvfp4)
'''


class AnchorDrift(RuntimeError):
    pass


def plan_patch(vllm_root: str) -> dict[str, tuple[str, list[str]]]:
    """New text of every file with seams, and the labels applied / already present.
    Raises AnchorDrift naming every seam whose anchor is not found exactly once."""
    texts: dict[str, str] = {}
    done: dict[str, list[str]] = {}
    drift = []
    for seam in SEAMS:
        path = os.path.join(vllm_root, seam.path)
        if path not in texts:
            if not os.path.isfile(path):
                drift.append(f"{seam.path} ({seam.label}): file missing")
                continue
            with open(path) as f:
                texts[path] = f.read()
            done[path] = []
        s = texts[path]
        if seam.new in s:
            done[path].append(f"{seam.label}: already patched")
            continue
        n = s.count(seam.old)
        if n != 1:
            drift.append(f"{seam.path} ({seam.label}): anchor found {n} times")
            continue
        texts[path] = s.replace(seam.old, seam.new, 1)
        done[path].append(f"{seam.label}: patched")
    if drift:
        raise AnchorDrift("ANCHOR DRIFT -- nothing written:\n  " + "\n  ".join(drift))
    return {p: (texts[p], done[p]) for p in texts}


def _write_atomic(path: str, text: str) -> None:
    d = os.path.dirname(path)
    fd, tmp = tempfile.mkstemp(dir=d, prefix=".nvfp4kv-")
    try:
        with os.fdopen(fd, "w") as f:
            f.write(text)
        mode = os.stat(path).st_mode if os.path.exists(path) else 0o644
        os.chmod(tmp, mode & 0o7777)
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise


def apply(vllm_root: str, check_only: bool = False) -> list[str]:
    """Patch the vLLM tree at ``vllm_root`` (the package directory); returns log lines."""
    plans = plan_patch(vllm_root)
    log = []
    for path, (text, labels) in plans.items():
        log += [f"[nvfp4-kv] {os.path.relpath(path, vllm_root)}: {x}" for x in labels]
        if not check_only and any(x.endswith(": patched") for x in labels):
            _write_atomic(path, text)
    shim = os.path.join(vllm_root, RUNTIME_MODULE)
    if not check_only:
        _write_atomic(shim, RUNTIME_SHIM)
    log.append(f"[nvfp4-kv] {RUNTIME_MODULE}: {'would be installed' if check_only else 'installed'}")
    return log


def default_vllm_root() -> str:
    import importlib.util

    spec = importlib.util.find_spec("vllm")
    if spec is None or not spec.submodule_search_locations:
        raise SystemExit("[nvfp4-kv] vllm is not importable here; pass --vllm-root")
    return list(spec.submodule_search_locations)[0]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--vllm-root", help="the vllm package directory (default: the importable vllm)")
    ap.add_argument("--check", action="store_true", help="verify every anchor, write nothing")
    args = ap.parse_args(argv)
    root = args.vllm_root or default_vllm_root()
    try:
        for line in apply(root, check_only=args.check):
            print(line)
    except AnchorDrift as e:
        print(f"[nvfp4-kv] {e}", file=sys.stderr)
        return 1
    print("[nvfp4-kv] all seams " + ("verified" if args.check else "patched"))
    return 0


if __name__ == "__main__":
    sys.exit(main())
