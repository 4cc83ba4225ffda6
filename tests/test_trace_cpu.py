"""CPU: the host side of the device phase trace (``blackwell_ops.device.Trace``).

The records a traced launch writes (u64 rec[16] = {gridid, blockIdx.x | gridDim.x << 32,
kernel id | smid << 32, stamp[0..12]}) are built here by hand, two launches of two kernels
interleaved, and read back through ``Trace.launches``: records are grouped by grid id, ordered
by CTA, named by kernel id with that kernel's phase names, and ``phases_us`` gives each phase's
end (max over CTAs) from the first CTA start, with first and median CTA.
"""
import pytest

torch = pytest.importorskip("torch")


def _record(grid, cta, ctas, kid, sm, stamps):
    r = [grid, cta | (ctas << 32), kid | (sm << 32)] + list(stamps) + [0] * (13 - len(stamps))
    return r


def _trace(records):
    from blackwell_ops.device import RECORD_WORDS, Trace

    tr = Trace.__new__(Trace)  # no device buffer: the records are filled in on the host
    tr.buf = torch.tensor(records, dtype=torch.int64).view(-1)
    tr.count = len(records)
    assert tr.buf.numel() == tr.count * RECORD_WORDS
    return tr


def test_trace_groups_names_and_phase_times():
    from blackwell_ops.device import PHASES, REQUANT_PHASES

    t0 = 1_000_000
    rec = [
        # requant launch (grid 7, two CTAs), written out of CTA order
        _record(7, 1, 2, 3, 5, [t0 + 500, t0 + 4500, t0 + 20000, t0 + 26000, t0 + 28000, t0 + 47000,
                                t0 + 19000, t0 + 45000, t0 + 19500, t0 + 46000]),
        # GEMM launch (grid 9, two CTAs), later
        _record(9, 0, 2, 1, 0, [t0 + 60000, t0 + 62000, t0 + 70000, t0 + 71000]),
        _record(7, 0, 2, 3, 4, [t0, t0 + 4000, t0 + 21000, t0 + 26500, t0 + 29000, t0 + 48000,
                                t0 + 18000, t0 + 44000, t0 + 18500, t0 + 45500]),
        _record(9, 1, 2, 1, 1, [t0 + 60200, t0 + 63000, t0 + 69000, t0 + 72000]),
    ]
    ls = _trace(rec).launches()
    assert [l.kernel for l in ls] == ["lora_requant_coop", "w8a16_persistent"]  # by first start
    req, gemm = ls
    assert req.grid_id == 7 and req.ctas == 2 and req.phases == REQUANT_PHASES
    assert req.stamps.shape == (2, len(REQUANT_PHASES))
    assert req.smid.tolist() == [4, 5]  # CTA order
    ph = req.phases_us()
    assert ph["cta_start_spread"] == 0.5
    assert ph["first_item"] == 4.5 and ph["first_item_first"] == 4.0
    assert ph["pass1_done"] == 21.0 and ph["barrier_passed"] == 26.5 and ph["pass2_done"] == 48.0
    assert ph["mma_done"] == 46.0 and ph["loads_issued"] == 45.0
    assert gemm.phases == PHASES and gemm.stamps.shape == (2, len(PHASES))
    g = gemm.phases_us()
    assert g["first_tile"] == 3.0 and g["mma_done"] == 10.0 and g["epilogue_done"] == 12.0
    assert "reduce_done" not in g  # a phase no CTA reached is left out
