"""The fused activation epilogues compute Sigmoid/SiLU with a branch-free
reciprocal (hardware approximation + Newton + Markstein correction) in place
of the IEEE division the reference performs (VectorMath.cs:70-77). It must
return the same bits as 1/d for every divisor the epilogues can see:
d = 1 + exp(-x) with x clamped to [-87.3, 88.7], i.e. every float in
[1, 2^126). The check runs on the device over all 1 056 964 608 of them."""
from __future__ import annotations

import ctypes as C

import pytest

pytestmark = pytest.mark.gpu


def test_branch_free_reciprocal_equals_ieee_division_exhaustively(ctx):
    from onnxsharp_b200._lib import call

    bad = C.c_ulonglong(0)
    first = C.c_uint(0)
    call("osc_selfcheck_recip", ctx.handle, C.byref(bad), C.byref(first))
    assert bad.value == 0, f"{bad.value} mismatches, first at bits {first.value:#010x}"


def test_fast_epilogue_activation_within_parity_tolerance(ctx):
    """The tensor-core conv epilogues use hardware ex2/rcp for Sigmoid and SiLU.
    Over every finite float the result stays within 2e-6 of the exact
    restatement in the parity metric |d| / max(1, |ref|) (tolerance 1e-4)."""
    from onnxsharp_b200._lib import call

    sig = C.c_float(0)
    silu = C.c_float(0)
    call("osc_selfcheck_fast_act", ctx.handle, C.byref(sig), C.byref(silu))
    assert sig.value <= 2e-6, sig.value
    assert silu.value <= 2e-6, silu.value
