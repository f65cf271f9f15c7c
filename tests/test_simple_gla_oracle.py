"""Pin the simple-GLA oracle (GLA oracle on the K-broadcast scalar gate) against the
reference's simple-GLA Torch code (fixtures from ``tests/golden/make_simple_gla_golden.py``)."""
from __future__ import annotations

import numpy as np
import pytest

import simple_gla_cases as SC
from oracle import simple_gla_oracle as SO
from test_oracle import BWD_TOL, FWD_TOL, _close


@pytest.mark.parametrize("case", SC.SIMPLE_CASES, ids=lambda c: c["name"])
def test_simple_oracle_matches_reference(case):
    c, inp, fx = SC.load(case["name"])
    o, ht = SO.chunk_simple_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["g_gamma"], inp["scale"], inp["h0"],
                                    True, inp["cu"], inp["C"])
    _close("o", o, fx["o"], **FWD_TOL)
    _close("ht", ht * SC.pad_decay(inp), fx["ht"], **FWD_TOL)
    dq, dk, dv, dg, dh0 = SO.chunk_simple_gla_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["g_gamma"],
                                                  inp["scale"], inp["h0"], inp["do"], inp["dht"], inp["cu"], inp["C"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        _close(nm, got, fx[nm], **BWD_TOL)
    assert (dg is None) == ("dg" not in fx)
    if dg is not None:
        _close("dg", dg, fx["dg"], **BWD_TOL)
    assert (dh0 is None) == ("dh0" not in fx)
    if dh0 is not None:
        _close("dh0", dh0, fx["dh0"], **BWD_TOL)


@pytest.mark.parametrize("case", SC.SIMPLE_CASES[:6], ids=lambda c: c["name"])
def test_simple_naive_equals_chunk(case):
    """The step-loop definition (tops/ops/simple_gla/naive.py) equals the chunked form."""
    c, inp, fx = SC.load(case["name"])
    B, T, H, K = inp["q"].shape
    g4 = None if inp["g"] is None else inp["g"][..., None]
    gg4 = None if inp["g_gamma"] is None else inp["g_gamma"].reshape(1, 1, H, 1)
    o, ht = SO.simple_gla_naive(inp["q"], inp["k"], inp["v"], g4, gg4, inp["scale"], inp["h0"], True, inp["cu"])
    _close("naive o", o, fx["o"], **FWD_TOL)
    _close("naive ht", ht * SC.pad_decay(inp), fx["ht"], **FWD_TOL)
