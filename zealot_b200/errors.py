"""ZealotError mirror (src/error.rs:4-47) and the zl_status -> exception map."""
from __future__ import annotations

from . import _capi


class ZealotError(RuntimeError):
    """Base of every error the library reports (ZealotError in the reference)."""
    status = -1


class InvalidArgument(ZealotError):
    status = 1


class CudaError(ZealotError):
    status = 2


class OobBlockError(ZealotError):
    """A block id or slot outside the pool reached a kernel (device status word)."""
    status = 3


class DeviceTimeout(ZealotError):
    """A bounded device wait ran out (device status word)."""
    status = 4


class NcclError(ZealotError):
    status = 5


class PeerLost(NcclError):
    """A peer rank left the job or stopped answering; found on the host before
    any collective of the step was launched (dist.PeerWatch)."""


class Unsupported(ZealotError):
    status = 6


class OutOfBlocks(ZealotError):
    status = 7


class StaleHandle(ZealotError):
    status = 8


class BlockNotAllocated(ZealotError):
    status = 9


class InvalidBlockSize(ZealotError):
    status = 10


class InternalError(ZealotError):
    status = 11


class SequenceTooLong(ZealotError):
    status = 12


_BY_STATUS = {c.status: c for c in (InvalidArgument, CudaError, OobBlockError, DeviceTimeout,
                                    NcclError, Unsupported, OutOfBlocks, StaleHandle,
                                    BlockNotAllocated, InvalidBlockSize, InternalError,
                                    SequenceTooLong)}


def check(status: int) -> None:
    """Raises the mapped exception for a non-zero zl_status."""
    if status == 0:
        return
    lib = _capi.load()
    msg = (lib.zl_last_error() or b"").decode(errors="replace")
    raise _BY_STATUS.get(status, ZealotError)(f"[zl_status {status}] {msg}")
