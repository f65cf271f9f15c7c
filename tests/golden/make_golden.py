"""Generate the golden fixtures ``tests/golden/{chunk,rec}_*.npz`` from the REFERENCE.

Run where the reference tree is available (read-only is enough):

    TOPS_REF=/path/to/pallas-kernel python tests/golden/make_golden.py

The reference's operators are JAX/Pallas-TPU and JAX cannot be installed here, so
the outputs come from the reference's own Torch CPU restatement under
``tests/src/ops/gla`` -- the gold its Pallas tests compare against
(``tests/ops/gla/test_pallas_chunk_gla.py:16,211-215``,
``tests/ops/gla/test_pallas_chunk_bwd.py:15,124-153``).  The reference's tests
pin JAX == that Torch code at 1e-5 (fwd) / 2e-5..5e-5 (bwd) / 1e-4 (recurrent).

Inputs are not stored: ``cases.py`` regenerates them from the seed and the
fixture keeps their SHA-256 digest.  Nothing at test time needs the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases as C  # noqa: E402

REF = os.environ.get("TOPS_REF", "/root/reference")


def _import_ref():
    sys.path.insert(0, REF)
    from tests.src.ops.gla import chunk as ref_chunk  # type: ignore
    from tests.src.ops.gla.fused_recurrent import fused_recurrent_gla, fused_recurrent_gla_bwd  # type: ignore
    from tests.src.ops.gla.naive import naive_recurrent_gla  # type: ignore
    return ref_chunk, fused_recurrent_gla, fused_recurrent_gla_bwd, naive_recurrent_gla


def _t(x):
    import torch
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x))


def make_chunk(ref_chunk):
    import torch
    for c in C.CHUNK_CASES:
        inp = C.chunk_inputs(c)
        cu_t = torch.tensor(inp["cu"], dtype=torch.long) if inp["cu"] else None
        gc, A, h, ht, o = ref_chunk.chunk_gla_fwd(
            _t(inp["q"]), _t(inp["k"]), _t(inp["v"]), _t(inp["g"]), g_cumsum=None, scale=inp["scale"],
            initial_state=_t(inp["h0"]), output_final_state=True, cu_seqlens=cu_t, chunk_size=inp["C"])
        out = dict(o=o.numpy(), ht=ht.numpy())
        small = h.numel() <= 60000 and A.numel() <= 60000
        if small:
            out.update(g_cumsum=gc.numpy(), A=A.numpy(), h=h.numpy())
        if not c.get("fwd_only"):
            dq, dk, dv, dg, dh0 = ref_chunk.chunk_gla_bwd(
                _t(inp["q"]), _t(inp["k"]), _t(inp["v"]), _t(inp["g"]), None, inp["scale"], _t(inp["h0"]),
                None, None, _t(inp["do"]), _t(inp["dht"]), cu_seqlens=cu_t, chunk_size=inp["C"])
            out.update(dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy(), dg=dg.numpy())
            if dh0 is not None:
                out["dh0"] = dh0.numpy()
            if small:
                dh, _ = ref_chunk.chunk_bwd_dh(
                    _t(inp["q"]), _t(inp["k"]), _t(inp["v"]), gc, _t(inp["do"]), h0=_t(inp["h0"]),
                    dht=_t(inp["dht"]), scale=inp["scale"], cu_seqlens=cu_t, chunk_size=inp["C"]) \
                    if inp["q"].shape[1] % inp["C"] == 0 and (not inp["cu"] or all(x % inp["C"] == 0 for x in inp["cu"])) \
                    else (None, None)
                if dh is not None:
                    out["dh"] = dh.numpy()
        out["input_digest"] = np.array(C.input_digest(inp, C.CHUNK_KEYS))
        np.savez_compressed(C.GOLDEN_DIR / f"chunk_{c['name']}.npz", **out)
        print("wrote chunk", c["name"])


def make_rec(frg, frg_bwd, naive):
    for c in C.REC_CASES:
        inp = C.rec_inputs(c)
        import torch
        cu_t = torch.tensor(inp["cu"], dtype=torch.long) if inp["cu"] else None
        o, ht = frg(_t(inp["q"]), _t(inp["k"]), _t(inp["v"]), gk=_t(inp["gk"]), gv=_t(inp["gv"]),
                    scale=inp["scale"], initial_state=_t(inp["h0"]), output_final_state=True,
                    reverse=inp["reverse"], cu_seqlens=cu_t)
        dq, dk, dv, dgk, dgv, dh0 = frg_bwd(
            _t(inp["q"]), _t(inp["k"]), _t(inp["v"]), gk=_t(inp["gk"]), gv=_t(inp["gv"]), o=o,
            do=_t(inp["do"]), dht=_t(inp["dht"]), scale=inp["scale"], initial_state=_t(inp["h0"]),
            reverse=inp["reverse"], cu_seqlens=cu_t)
        out = dict(o=o.numpy(), ht=ht.numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy())
        for nm, x in (("dgk", dgk), ("dgv", dgv), ("dh0", dh0)):
            if x is not None:
                out[nm] = x.numpy()
        if inp["gk"] is not None and inp["gv"] is None and not inp["reverse"]:
            on, hn = naive(_t(inp["q"]), _t(inp["k"]), _t(inp["v"]), _t(inp["gk"]), scale=inp["scale"],
                           initial_state=_t(inp["h0"]), output_final_state=True, cu_seqlens=cu_t)
            out["naive_o"], out["naive_ht"] = on.numpy(), hn.numpy()
        out["input_digest"] = np.array(C.input_digest(inp, C.REC_KEYS))
        np.savez_compressed(C.GOLDEN_DIR / f"rec_{c['name']}.npz", **out)
        print("wrote rec", c["name"])


if __name__ == "__main__":
    ref_chunk, frg, frg_bwd, naive = _import_ref()
    make_chunk(ref_chunk)
    make_rec(frg, frg_bwd, naive)
