"""libcbx_ops: B200 (sm_100a) fused per-layer elementwise ops of the Chatterbox
TTS engine (T3 / S3Gen-CFM / HiFT), behind a C ABI (include/cbx_ops.h).

- ``chatterbox_amdvulkan_b200.ops``   torch-facing wrappers named after the
  engine's layer helpers (one libcbx_ops kernel per call, current stream);
- ``chatterbox_amdvulkan_b200.shard`` row/utterance sharding across GPUs and
  the NCCL result gather;
- ``chatterbox_amdvulkan_b200.build`` nvcc build of libcbx_ops.so (in-tree).
"""
from ._lib import LIB_PATH, CbxError, load  # noqa: F401

__all__ = ["LIB_PATH", "CbxError", "load"]
