"""Parity gates shared by the GPU tests (imported by them; not a test module)."""

import math

from oracle import compare_outputs


def no_worse_than_reference_rounding(ref32, ours, ref_style, what):
    """Gate for 16-bit results whose reference-style evaluation itself misses the
    predicate: ``ours`` and ``ref_style`` (the reference's own 16-bit storage
    points) are both compared with fp32 ``ref32`` under the reference predicate
    (abs 2e-3 OR rel 2e-2).  If ref_style passes, ours must pass; otherwise ours
    may fail at most 1.25x as many elements (plus one per million) and its mean
    and maximum errors may exceed ref_style's by at most 15% and 50%."""
    r_ours = compare_outputs(ref32, ours)
    r_ref = compare_outputs(ref32, ref_style)
    print(f"\n{what}: ours vs fp32 {r_ours}; reference 16-bit storage vs fp32 {r_ref}")
    if r_ref.passed:
        assert r_ours.passed, f"{what}: {r_ours}"
        return r_ours, r_ref
    slack = math.ceil(1e-6 * r_ours.total_elements)
    assert r_ours.failed_elements <= math.ceil(1.25 * r_ref.failed_elements) + slack, (what, r_ours, r_ref)
    assert r_ours.mean_abs_error <= 1.15 * r_ref.mean_abs_error + 1e-6, (what, r_ours, r_ref)
    assert r_ours.max_abs_error <= 1.5 * r_ref.max_abs_error + 1e-4, (what, r_ours, r_ref)
    return r_ours, r_ref
