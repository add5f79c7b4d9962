"""B200-native (sm_100a) NVFP4 paged KV-cache path: quantize-on-append, 656-byte compat
gather, and a fused NVFP4 gather + MLA decode kernel on tcgen05, behind the module surface
of the reference's glm53_nvfp4_runtime (see ``glm53_nvfp4_runtime``)."""

__all__ = ["glm53_nvfp4_runtime", "partition"]
