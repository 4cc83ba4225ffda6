"""Device-side status, wait limit and phase trace of libbw_ops.so.

The reference's operators fail only through ``TORCH_CHECK`` on the host; the
kernels here also have spin waits (mbarrier pipelines, the fused all-gather's
wait for its peers' output words, the requantiser's grid barrier), every one
bounded.  A wait that
runs out records its site in a device status word and its kernel unwinds
without finishing its output.  This module turns that into Python errors:

* ``check(device)`` synchronises, reads the status and raises
  ``DeviceTimeoutError`` (a ``RuntimeError``) if any wait ran out since the last
  check, after clearing the status and re-zeroing the cached GEMM workspaces
  (an aborted split-K reduction can leave a tile counter non-zero).
* ``set_wait_limit(seconds)`` / ``wait_limit()`` set and read the bound of every
  spin wait on a device (default 4 s).
* ``Trace`` records, per CTA of each traced kernel launch, globaltimer stamps of
  its phases, so a caller can see which phase bounds a step.  The W8A16 GEMM:
  start, first weight tile landed, last MMA complete, epilogue done, the
  deferred stream-K reductions done, and for the fused all-gather: call epoch
  read, every peer's outputs received; and when the preceding kernel completed.
  The fused merge + requantisation: start, first accumulator of each pass
  ready, pass 1 done (grid-barrier arrival), grid barrier passed, pass 2 done,
  and when its TMA producer and MMA issuer finished each pass.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import BW_ERR_DEVICE_TIMEOUT, BW_OK, BwError, check as _check, lib, stream_ptr


class DeviceTimeoutError(BwError):
    """A kernel's bounded wait ran out (a peer never arrived, or a pipeline stalled)."""


def _dev(device) -> torch.device:
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.index is None:
        return torch.device("cuda", torch.cuda.current_device())
    return device


def status(device=None, clear: bool = False) -> int:
    """Synchronise ``device``'s current stream and return the wait-site id of the
    first expired wait since the last clear (0: none)."""
    dev = _dev(device)
    detail = ctypes.c_int(0)
    with torch.cuda.device(dev):
        st = lib.bw_device_status(1 if clear else 0, ctypes.byref(detail), stream_ptr(dev))
    if st not in (BW_OK, BW_ERR_DEVICE_TIMEOUT):
        _check(st, "device status")
    return detail.value


def check(device=None, op: str = "blackwell_ops") -> None:
    """Raise ``DeviceTimeoutError`` if a bounded wait of a kernel on ``device`` ran out.

    Clears the status and re-zeroes the cached GEMM and requantisation workspaces first,
    so the next call starts clean.  Synchronises the device's current stream."""
    site = status(device, clear=True)
    if site:
        from .cuda import reset_workspaces as reset_requant
        from .kernels.int8_gemm import reset_workspaces

        reset_workspaces()
        reset_requant()
        torch.cuda.synchronize(_dev(device))
        err = DeviceTimeoutError(BW_ERR_DEVICE_TIMEOUT, op)
        err.site = site
        raise err


def set_wait_limit(seconds: float, device=None) -> None:
    """Bound of every spin wait in this library's kernels on ``device``."""
    ns = int(seconds * 1e9)
    with torch.cuda.device(_dev(device)):
        _check(lib.bw_set_wait_limit_ns(ctypes.c_uint64(ns)), "set_wait_limit")


def wait_limit(device=None) -> float:
    ns = ctypes.c_uint64(0)
    with torch.cuda.device(_dev(device)):
        _check(lib.bw_get_wait_limit_ns(ctypes.byref(ns)), "wait_limit")
    return ns.value / 1e9


PHASES = ("start", "first_tile", "mma_done", "epilogue_done", "reduce_done", "epoch_read", "gather_done",
          "predecessor_done")
# the fused merge + requantisation kernel's phases: its two passes over the items, the grid
# barrier between them, and when its TMA producer and first MMA issuer finished each pass
REQUANT_PHASES = ("start", "first_item", "pass1_done", "barrier_passed", "pass2_first_item", "pass2_done",
                  "pass1_loads_issued", "loads_issued", "mma_pass1_done", "mma_done")
RECORD_WORDS = 16
KERNEL_IDS = {1: "w8a16_persistent", 2: "w8a16_persistent_swiglu", 3: "lora_requant_coop"}
KERNEL_PHASES = {3: REQUANT_PHASES}


@dataclass
class Launch:
    grid_id: int
    kernel: str
    ctas: int
    stamps: torch.Tensor  # [ctas, len(phases)] int64 ns, 0 = not reached
    smid: torch.Tensor    # [ctas] SM of each CTA
    phases: tuple = PHASES

    def phases_us(self) -> dict:
        """Phase ends relative to the first CTA start, in microseconds (max over CTAs), and
        the spread of CTA start times."""
        s = self.stamps.double()
        t0 = float(s[:, 0][s[:, 0] > 0].min())
        out = {"cta_start_spread": round((float(s[:, 0].max()) - t0) / 1e3, 3)}
        for i, name in enumerate(self.phases[1:], start=1):
            col = s[:, i][s[:, i] > 0]
            if col.numel():
                out[name] = round((float(col.max()) - t0) / 1e3, 3)
                if col.numel() > 1:  # first CTA and median CTA: the spread shows load balance
                    out[name + "_first"] = round((float(col.min()) - t0) / 1e3, 3)
                    out[name + "_median"] = round((float(col.median()) - t0) / 1e3, 3)
        return out


class Trace:
    """Collects the phase stamps of traced kernel launches on one device.

    with Trace(records=4096) as tr:
        ... launches ...
    launches = tr.launches()
    """

    def __init__(self, records: int = 4096, device=None):
        self.dev = _dev(device)
        self.buf = torch.zeros(records * RECORD_WORDS, dtype=torch.int64, device=self.dev)

    def __enter__(self):
        torch.cuda.synchronize(self.dev)
        with torch.cuda.device(self.dev):
            _check(lib.bw_trace_enable(self.buf.data_ptr(), self.buf.numel() * 8), "trace enable")
        return self

    def __exit__(self, *exc):
        torch.cuda.synchronize(self.dev)
        n = ctypes.c_uint(0)
        with torch.cuda.device(self.dev):
            _check(lib.bw_trace_records(ctypes.byref(n)), "trace records")
            _check(lib.bw_trace_enable(None, 0), "trace disable")
        self.count = n.value

    def launches(self) -> list[Launch]:
        rec = self.buf[: self.count * RECORD_WORDS].view(-1, RECORD_WORDS).cpu()
        by_grid: dict[int, list] = {}
        for r in rec:
            by_grid.setdefault(int(r[0]), []).append(r)
        out = []
        for gid, rows in by_grid.items():
            rows = torch.stack(rows)
            ctas = int(rows[0, 1]) >> 32
            order = torch.argsort(rows[:, 1] & 0xFFFFFFFF)
            kid = int(rows[0, 2]) & 0xFFFFFFFF
            names = KERNEL_PHASES.get(kid, PHASES)
            out.append(Launch(gid, KERNEL_IDS.get(kid, str(kid)), ctas, rows[order, 3:3 + len(names)],
                              (rows[order, 2] >> 32) & 0xFFFFFFFF, names))
        out.sort(key=lambda l: int(l.stamps[:, 0][l.stamps[:, 0] > 0].min()))
        return out
