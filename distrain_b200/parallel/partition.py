"""SM partition for the coordinator's merge (``csrc/kernels/partition.cu``).

The reference runs its merge on the coordinator's own process and device
(``coordinator/src/aggregation.rs:346-349,380``); in a training box the coordinator shares every GPU
with a training node, so the merge kernels are given a partition of their own: a green context that
owns ``sms`` SMs (rounded up by the driver to its granularity) and a high-priority stream in it. The
merge's kernels then never occupy more than that group of SMs while the node keeps training on the
rest; with ``sms = 0`` the merge uses an ordinary priority stream over the whole GPU.
"""
from __future__ import annotations

import ctypes
import torch


class SmPartition:
    """A green context of at least ``sms`` SMs on ``device`` and a stream in it (``self.stream``, a
    ``torch.cuda.ExternalStream`` usable with ``torch.cuda.stream`` and by the kernel library)."""

    def __init__(self, device, sms: int, priority: int = -100):
        from ..ops import _lib
        from ..ops._lib import c_int, c_void
        self.L = _lib.lib()
        pv, pi = ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int)
        _lib.register("dt_sm_partition_create", [c_int, c_int, c_int, pv, pv, pi, pi])
        _lib.register("dt_sm_partition_destroy", [c_void, c_void])
        self.device = torch.device(device)
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        s, h = ctypes.c_void_p(), ctypes.c_void_p()
        got, total = ctypes.c_int(), ctypes.c_int()
        with torch.cuda.device(idx):
            # the driver clamps the priority into the device's range
            rc = self.L.dt_sm_partition_create(idx, int(sms), int(priority), ctypes.byref(s), ctypes.byref(h),
                                               ctypes.byref(got), ctypes.byref(total))
        if rc != 0:
            raise RuntimeError(f"SM partition of {sms} SMs on cuda:{idx} failed (code {rc})")
        self._handle, self._raw = h.value, s.value
        self.sms, self.total_sms = got.value, total.value
        self.stream = torch.cuda.ExternalStream(self._raw, device=torch.device("cuda", idx))

    def close(self):
        """Waits for the partition's work. The green context itself lives until the process exits: torch's
        allocators keep events recorded on its stream (pinned staging copies, cross-stream frees) and
        record more when those blocks are released, which must not find the stream destroyed."""
        self.stream.synchronize()


_PARTITIONS = {}


def partition(device, sms: int) -> SmPartition:
    """The process's SM partition of ``sms`` SMs on ``device`` (created once, shared by later callers)."""
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), int(sms))
    if key not in _PARTITIONS:
        _PARTITIONS[key] = SmPartition(torch.device("cuda", key[0]), sms)
    return _PARTITIONS[key]


def merge_stream(device, sms: int) -> torch.cuda.Stream:
    """The stream the coordinator's merge kernels run on: the stream of a green-context partition of
    ``sms`` SMs when ``sms > 0``, else a top-priority stream over the whole device."""
    if sms and sms > 0:
        return partition(device, sms).stream
    return torch.cuda.Stream(device=device, priority=-100)
