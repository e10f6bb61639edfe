"""Source-level guards for the CUDA code (CPU, no build needed).

* No bulk or tensor copy uses cluster multicast: multi-GPU runs must never reach a
  multicast load whose source could be another GPU's memory, so the library has none.
* No batched memcpy entry point of the CUDA runtime or driver is used: one
  cudaMemcpyAsync per copy (or a gather kernel) instead.
* Every spin on an mbarrier goes through the bounded helpers of tma_util.cuh or the
  kernels' own bounded waits (a try_wait loop with a %globaltimer limit).

The patterns are assembled from pieces so that this file itself names none of them.
"""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCES = sorted(glob.glob(os.path.join(ROOT, "xe2x2_b200", "csrc", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "xe2x2_b200", "csrc", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "xe2x2_b200", "csrc", "*.h")))


def _code_lines(path):
    """Source lines with // comments removed (comments may describe what is absent)."""
    with open(path) as f:
        for n, line in enumerate(f, 1):
            yield n, line.split("//", 1)[0]


def test_sources_found():
    assert len(SOURCES) >= 10


def test_no_multicast_copies():
    """The multicast qualifier appears on no code line at all (an inline-asm string split over
    adjacent literals would otherwise hide it from a same-line check)."""
    mc = "multi" + "cast"
    bad = [(os.path.basename(p), n) for p in SOURCES for n, line in _code_lines(p) if mc in line.lower()]
    assert not bad, bad


def test_no_batched_memcpy_entry_points():
    names = [pre + "Memcpy" + mid + "Batch" + "Async" for pre in ("cuda", "cu") for mid in ("", "3D")]
    bad = [(os.path.basename(p), n, name) for p in SOURCES for n, line in _code_lines(p) for name in names
           if name in line]
    assert not bad, bad


def test_mbarrier_try_wait_only_inside_bounded_helpers():
    """try_wait appears in the helper that wraps it; every loop around a try_wait helper
    call also reads the global timer (or the CTA's abort flag set by one that does)."""
    uses = []
    for p in SOURCES:
        text = open(p).read()
        for m in re.finditer(r"while\s*\(\s*!\s*mbar_try_wait\([^)]*\)\s*\)", text):
            body = text[m.end():m.end() + 400]
            uses.append((os.path.basename(p), "global_ns" in body or "abort_flag" in body))
        # the suspending form: the loop that calls it reads the global timer and gives up
        for m in re.finditer(r"for\s*\(\s*;\s*;\s*\)\s*\{", text):
            body = text[m.end():m.end() + 400]
            if "mbar_try_wait_suspend(" in body:
                uses.append((os.path.basename(p), "global_ns" in body and "return false" in body))
    assert uses, "expected bounded waits built on mbar_try_wait"
    assert all(ok for _, ok in uses), uses
