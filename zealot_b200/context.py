"""GpuContext: the library context bound to one device (src/gpu_context.rs:16-52)."""
from __future__ import annotations

import ctypes

from . import _capi
from .errors import check

GQA_GROUPED = 0  # kv = h / (H / Hkv)   (paged_attention.cu:32)
GQA_MODULO = 1   # kv = h % Hkv         (model_runner_cpu.rs:295)
# zl_ctx_set_flags: block tables, seq_lens and token ranges of later decode calls
# are written before the kernel that precedes the decode on its stream starts
CTX_INPUTS_AHEAD = 1

F32 = 0
BF16 = 1


def dtype_code(t) -> int:
    import torch
    if t == torch.float32:
        return F32
    if t == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {t}: the kernels take float32 or bfloat16")


def ptr(x) -> int:
    """Device address of a torch tensor (or an int address passed through)."""
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return x.data_ptr()


class _DeviceArray:
    """Minimal __cuda_array_interface__ holder so torch can view library-owned memory."""

    def __init__(self, address: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(address), False), "version": 3,
                                         "strides": None}


def device_view(address: int, shape, dtype):
    """Zero-copy torch view of device memory the library owns (pools, block tables)."""
    import torch
    typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.bfloat16: "<V2"}[dtype]
    if dtype == torch.bfloat16:
        t = torch.as_tensor(_DeviceArray(address, shape, "<i2"), device="cuda")
        return t.view(torch.bfloat16)
    return torch.as_tensor(_DeviceArray(address, shape, typestr), device="cuda")


def current_stream(device: int) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


class GpuContext:
    """Owns a zl_ctx: device binding, device status word, split-KV workspace."""

    def __init__(self, device: int = 0, workspace_bytes: int = 0):
        self.lib = _capi.load()
        self.device = device
        cfg = _capi.zl_ctx_cfg(device, workspace_bytes)
        h = ctypes.c_void_p()
        check(self.lib.zl_ctx_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.handle = h

    def stream(self, stream=None) -> int:
        if stream is None:
            return current_stream(self.device)
        return stream if isinstance(stream, int) else stream.cuda_stream

    def check_status(self, stream=None) -> None:
        """Synchronises the stream and raises if a kernel flagged a bad block
        id (OobBlockError) or a timed-out wait (DeviceTimeout)."""
        check(self.lib.zl_check_status(self.handle, self.stream(stream)))

    def launch_count(self) -> int:
        return int(self.lib.zl_launch_count(self.handle))

    def set_flags(self, flags: int) -> None:
        """zl_ctx_set_flags: CTX_INPUTS_AHEAD lets the decode kernel read its
        tables and lengths before waiting for the preceding kernel on its stream
        (only when they were written before that kernel started)."""
        check(self.lib.zl_ctx_set_flags(self.handle, flags))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.zl_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
