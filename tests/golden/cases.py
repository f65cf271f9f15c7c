"""Case matrix and seeded input generation shared by ``make_golden.py`` and the tests.

The fixtures store the reference's outputs plus a SHA-256 digest of the inputs;
the tests regenerate the inputs from the seed with :func:`chunk_inputs` /
:func:`rec_inputs` and check the digest before comparing, so a change in the
generator can never silently pair new inputs with old outputs.

Case shapes follow the reference's own test matrices
(``tests/ops/gla/test_pallas_chunk_gla.py:24-126``,
``tests/ops/gla/test_pallas_chunk_bwd.py:20-80``,
``tests/ops/gla/test_pallas_fused_recurrent.py:26-132``) plus BASELINE config 1.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

GOLDEN_DIR = Path(__file__).resolve().parent

CHUNK_CASES = [
    dict(name="std", B=2, T=32, H=4, K=32, V=64, seed=42, C=16),
    dict(name="std_h0", B=2, T=32, H=4, K=32, V=64, seed=13, C=16, h0=True),
    dict(name="std_dht", B=2, T=32, H=4, K=32, V=64, seed=14, C=16, dht=True),
    dict(name="t128", B=1, T=128, H=2, K=64, V=128, seed=7, C=16),
    dict(name="k16v128", B=2, T=32, H=4, K=16, V=128, seed=20, C=16),
    dict(name="k128v16", B=2, T=32, H=4, K=128, V=16, seed=21, C=16),
    dict(name="t1", B=1, T=1, H=2, K=32, V=64, seed=30, C=16),
    dict(name="t3", B=1, T=3, H=2, K=32, V=64, seed=31, C=16),
    dict(name="t37", B=2, T=37, H=4, K=16, V=32, seed=40, C=16),
    dict(name="t100_h0_dht", B=1, T=100, H=2, K=32, V=64, seed=42, C=16, h0=True, dht=True),
    dict(name="small_scale", B=2, T=32, H=2, K=8, V=16, seed=70, C=16, scale=0.1),
    dict(name="var_eq", B=1, T=32, H=4, K=32, V=64, seed=7, C=16, cu=[0, 16, 32]),
    dict(name="var_ragged_h0_dht", B=1, T=50, H=2, K=16, V=32, seed=602, C=16, cu=[0, 13, 37, 50],
         h0=True, dht=True),
    dict(name="var_ragged_h0", B=1, T=45, H=2, K=32, V=64, seed=604, C=16, cu=[0, 20, 45], h0=True),
    dict(name="var_many", B=1, T=96, H=2, K=16, V=32, seed=30, C=16, cu=[0, 16, 32, 48, 64, 80, 96]),
    dict(name="c64", B=2, T=128, H=4, K=32, V=64, seed=502, C=64),
    dict(name="c32", B=2, T=64, H=4, K=32, V=64, seed=500, C=32),
    dict(name="c8_h0_dht", B=1, T=128, H=2, K=32, V=64, seed=501, C=8, h0=True, dht=True),
    dict(name="c4", B=1, T=64, H=2, K=32, V=64, seed=503, C=4),
    dict(name="c32_var", B=1, T=64, H=4, K=32, V=64, seed=510, C=32, cu=[0, 32, 64]),
    dict(name="long_h0", B=1, T=512, H=2, K=32, V=64, seed=304, C=16, h0=True),
    # BASELINE config 1 (forward-only CPU correctness case): B2 T256 H4 K64 V64 C64,
    # q,k,v ~ N(0,1), g = logsigmoid(N(0,1))/16, h0 = 0, seed 0.
    dict(name="cfg1", B=2, T=256, H=4, K=64, V=64, seed=0, C=64, gnorm=16.0, h0z=True, fwd_only=True),
    # 128/256-wide heads at the configs' gate normalisation
    dict(name="k128v256_c64", B=1, T=192, H=2, K=128, V=256, seed=900, C=64, gnorm=16.0, h0=True, dht=True),
]

REC_CASES = [
    dict(name="gk", B=2, T=32, H=4, K=32, V=64, seed=42, gate="gk"),
    dict(name="gk_h0", B=2, T=32, H=4, K=32, V=64, seed=13, gate="gk", h0=True),
    dict(name="gv", B=2, T=32, H=4, K=32, V=64, seed=100, gate="gv"),
    dict(name="gkgv_h0", B=2, T=32, H=4, K=32, V=64, seed=133, gate="gk+gv", h0=True),
    dict(name="none", B=2, T=32, H=4, K=32, V=64, seed=102, gate="none"),
    dict(name="rev_h0", B=2, T=32, H=4, K=32, V=64, seed=111, gate="gk", reverse=True, h0=True),
    dict(name="t1_rev", B=1, T=1, H=2, K=16, V=32, seed=112, gate="gk", reverse=True),
    dict(name="t37", B=2, T=37, H=4, K=16, V=32, seed=40, gate="gk"),
    dict(name="k128v16", B=2, T=32, H=4, K=128, V=16, seed=21, gate="gk"),
    dict(name="var", B=1, T=23, H=2, K=16, V=32, seed=12, gate="gk", cu=[0, 7, 20, 23], h0=True),
    dict(name="var_rev_gkgv", B=1, T=48, H=4, K=32, V=64, seed=131, gate="gk+gv", cu=[0, 10, 24, 48],
         reverse=True, h0=True, dht=True),
    dict(name="var_unit", B=1, T=4, H=2, K=16, V=32, seed=20, gate="gk", cu=[0, 1, 2, 3, 4]),
    dict(name="scale_dht", B=2, T=32, H=4, K=32, V=64, seed=140, gate="gk", scale=0.1, h0=True, dht=True),
    # decode step, BASELINE config 2 distributions at reduced batch: bf16-representable q/k/v,
    # fp32 gk = logsigmoid(N)/16, h0 ~ N(0, 0.1)
    dict(name="decode", B=2, T=1, H=2, K=128, V=128, seed=2, gate="gk", gnorm=16.0, h0s=0.1, bf16=True),
    dict(name="k256", B=1, T=8, H=2, K=256, V=64, seed=77, gate="gk", h0=True),
]


def logsigmoid(x):
    return -np.logaddexp(0.0, -x)


def bf16_round(x):
    """Round-to-nearest-even fp32 -> bf16 -> fp32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def digest(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        if a is not None:
            h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def _qkvg(c, rng):
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    q = rng.standard_normal((B, T, H, K), dtype=np.float32)
    k = rng.standard_normal((B, T, H, K), dtype=np.float32)
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    g = (logsigmoid(rng.standard_normal((B, T, H, K)).astype(np.float32)) / c.get("gnorm", 1.0)).astype(np.float32)
    return q, k, v, g


def chunk_inputs(c):
    """Seeded inputs of a CHUNK_CASES entry -> dict of float32 arrays (None when absent)."""
    rng = np.random.default_rng(c["seed"])
    q, k, v, g = _qkvg(c, rng)
    B, H, K, V = c["B"], c["H"], c["K"], c["V"]
    cu = c.get("cu")
    N = len(cu) - 1 if cu else B
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("h0") else None
    if c.get("h0z"):
        h0 = np.zeros((N, H, K, V), np.float32)
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("dht") else None
    do = rng.standard_normal((B, c["T"], H, V), dtype=np.float32)
    return dict(q=q, k=k, v=v, g=g, h0=h0, dht=dht, do=do, cu=cu, C=c["C"],
                scale=c.get("scale", K ** -0.5))


def rec_inputs(c):
    """Seeded inputs of a REC_CASES entry."""
    rng = np.random.default_rng(c["seed"])
    q, k, v, g = _qkvg(c, rng)
    if c.get("bf16"):
        q, k, v = (bf16_round(x) for x in (q, k, v))
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    cu = c.get("cu")
    N = len(cu) - 1 if cu else B
    gate = c["gate"]
    gk = g if "gk" in gate else None
    gv = (logsigmoid(rng.standard_normal((B, T, H, V)).astype(np.float32)).astype(np.float32)
          if "gv" in gate else None)
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("h0") else None
    if c.get("h0s"):
        h0 = (rng.standard_normal((N, H, K, V), dtype=np.float32) * c["h0s"]).astype(np.float32)
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("dht") else None
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    if c.get("bf16"):
        do = bf16_round(do)
    return dict(q=q, k=k, v=v, gk=gk, gv=gv, h0=h0, dht=dht, do=do, cu=cu,
                scale=c.get("scale", K ** -0.5), reverse=bool(c.get("reverse", False)))


def input_digest(inp, keys):
    return digest(*[inp[k] for k in keys])


CHUNK_KEYS = ("q", "k", "v", "g", "h0", "dht", "do")
REC_KEYS = ("q", "k", "v", "gk", "gv", "h0", "dht", "do")


def load(kind, name):
    """Load a fixture and its regenerated inputs; raises if the inputs drifted."""
    cases = CHUNK_CASES if kind == "chunk" else REC_CASES
    c = next(x for x in cases if x["name"] == name)
    inp = chunk_inputs(c) if kind == "chunk" else rec_inputs(c)
    fx = dict(np.load(GOLDEN_DIR / f"{kind}_{name}.npz"))
    want = str(fx.pop("input_digest"))
    got = input_digest(inp, CHUNK_KEYS if kind == "chunk" else REC_KEYS)
    if want != got:
        raise RuntimeError(f"golden inputs for {kind}/{name} drifted: {got} != {want}")
    return c, inp, fx
