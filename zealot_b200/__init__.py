"""zealot_b200 -- the B200 (sm_100a) attention hot path of the Zealot engine.

The product is libzealot_attn.so (C ABI in include/zealot_attn.h, CUDA in
zealot_b200/csrc). This package is its Python host mirror, named after the
reference Rust interfaces it stands in for:

  GpuContext        src/gpu_context.rs:16-52
  CudaAttention     src/attention/cuda.rs:20-210 (paged_forward, forward_gpu)
                    + reshape_and_cache (src/kv_cache.rs:212-357)
  BlockManager      src/block_manager.rs:41-165
  KVCache           src/kv_cache.rs:51-357
  CudaModelRunner   src/cuda_runner.rs / the ModelRunner trait (src/engine.rs:15-37)
  Sequence          src/scheduler.rs:11-113 (the fields the runner reads)

Device memory is passed as torch tensors (plumbing only); every computation
runs in the library. Importing fails loudly if the library is not built.
"""
from . import _capi
from .errors import (ZealotError, InternalError, OutOfBlocks, StaleHandle, BlockNotAllocated,
                     InvalidBlockSize, SequenceTooLong, CudaError, OobBlockError, DeviceTimeout,
                     NcclError, PeerLost, Unsupported, InvalidArgument)
from .context import GpuContext, GQA_GROUPED, GQA_MODULO
from .attention import CudaAttention
from .kv_cache import BlockManager, BlockHandle, KVCache
from .runner import CudaModelRunner, Sequence, StepOut

lib = _capi.load()

__all__ = [
    "GpuContext", "CudaAttention", "BlockManager", "BlockHandle", "KVCache", "CudaModelRunner",
    "Sequence", "StepOut", "ZealotError", "InternalError", "OutOfBlocks", "StaleHandle",
    "BlockNotAllocated", "InvalidBlockSize", "SequenceTooLong", "CudaError", "OobBlockError",
    "DeviceTimeout", "NcclError", "PeerLost", "Unsupported", "InvalidArgument", "GQA_GROUPED", "GQA_MODULO",
    "lib",
]
