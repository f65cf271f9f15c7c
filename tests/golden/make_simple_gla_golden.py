"""Generate ``tests/golden/simple_*.npz`` from the REFERENCE's simple-GLA Torch CPU code.

    TOPS_REF=/path/to/pallas-kernel python tests/golden/make_simple_gla_golden.py

The reference's simple-GLA operators are JAX/Pallas; the fixtures come from its Torch CPU
restatement ``tests/src/ops/simple_gla/chunk.py`` (``chunk_simple_gla_fwd`` :329,
``chunk_simple_gla_bwd`` :784), the gold of its simple-GLA tests.  Inputs are not stored:
``simple_gla_cases.py`` regenerates them from the seed; the fixture keeps their digest.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import simple_gla_cases as S  # noqa: E402
from cases import digest  # noqa: E402

REF = os.environ.get("TOPS_REF", "/root/reference")


def main():
    import torch
    sys.path.insert(0, REF)
    from tests.src.ops.simple_gla import chunk as ref  # type: ignore

    t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x))
    for c in S.SIMPLE_CASES:
        inp = S.simple_inputs(c)
        cu = torch.tensor(inp["cu"], dtype=torch.long) if inp["cu"] else None
        _, _, _, ht, o = ref.chunk_simple_gla_fwd(t(inp["q"]), t(inp["k"]), t(inp["v"]), t(inp["g"]),
                                                  t(inp["g_gamma"]), inp["scale"], t(inp["h0"]), True,
                                                  cu_seqlens=cu, chunk_size=inp["C"])
        dq, dk, dv, dg, dh0 = ref.chunk_simple_gla_bwd(t(inp["q"]), t(inp["k"]), t(inp["v"]), t(inp["g"]),
                                                       t(inp["g_gamma"]), inp["scale"], t(inp["h0"]), t(inp["do"]),
                                                       t(inp["dht"]), cu_seqlens=cu, chunk_size=inp["C"])
        out = dict(o=o.numpy(), ht=ht.numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy())
        if dg is not None:
            out["dg"] = dg.numpy()
        if dh0 is not None:
            out["dh0"] = dh0.numpy()
        out["input_digest"] = np.array(digest(*[inp[k] for k in S.SIMPLE_KEYS]))
        np.savez_compressed(S.GOLDEN_DIR / f"simple_{c['name']}.npz", **out)
        print("wrote simple", c["name"])


if __name__ == "__main__":
    main()
