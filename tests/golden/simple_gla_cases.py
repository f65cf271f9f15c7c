"""Case matrix and seeded inputs for the simple-GLA fixtures (``simple_*.npz``).

Shapes follow the reference's simple-GLA test matrices
(``tests/ops/simple_gla/test_torch_simple_gla_bwd.py:48-76``,
``tests/ops/simple_gla/test_simple_gla.py:48+``): gate modes "g" (logsigmoid of N(0,1),
[B, T, H]), "gamma" (g_gamma = -|U(0,1)| * 0.5, [H]) and "both"; ragged T; h0 / dht;
chunk sizes 16..64; packed varlen.  Inputs are regenerated from the seed and checked
against the digest stored in each fixture.
"""
from __future__ import annotations

import numpy as np

from cases import GOLDEN_DIR, digest, logsigmoid

SIMPLE_CASES = [
    dict(name="gamma", B=2, T=64, H=4, K=32, V=64, seed=42, gate="gamma"),
    dict(name="gamma_k64v128", B=1, T=128, H=2, K=64, V=128, seed=7, gate="gamma"),
    dict(name="gamma_h0", B=2, T=64, H=4, K=32, V=64, seed=13, gate="gamma", h0=True),
    dict(name="gamma_h0_dht", B=2, T=64, H=4, K=32, V=64, seed=15, gate="gamma", h0=True, dht=True),
    dict(name="gamma_t100", B=2, T=100, H=4, K=32, V=64, seed=400, gate="gamma"),
    dict(name="g", B=2, T=64, H=4, K=32, V=64, seed=42, gate="g"),
    dict(name="g_h1", B=2, T=64, H=1, K=32, V=64, seed=10, gate="g"),
    dict(name="g_k16v128", B=2, T=64, H=4, K=16, V=128, seed=20, gate="g"),
    dict(name="g_h0_dht", B=2, T=64, H=4, K=32, V=64, seed=15, gate="g", h0=True, dht=True),
    dict(name="g_t100", B=2, T=100, H=4, K=32, V=64, seed=400, gate="g"),
    dict(name="g_c16", B=2, T=64, H=4, K=32, V=64, seed=500, gate="g", C=16),
    dict(name="both", B=1, T=128, H=2, K=64, V=128, seed=7, gate="both"),
    dict(name="both_h0_dht", B=2, T=64, H=4, K=32, V=64, seed=15, gate="both", h0=True, dht=True),
    dict(name="both_t256_c32", B=1, T=256, H=2, K=32, V=64, seed=300, gate="both", C=32),
    dict(name="g_var", B=1, T=96, H=2, K=32, V=64, seed=610, gate="g", cu=[0, 64, 96], h0=True, dht=True),
    dict(name="both_var_ragged", B=1, T=90, H=2, K=32, V=64, seed=611, gate="both", cu=[0, 17, 70, 90], h0=True),
    dict(name="g_k128v128", B=1, T=192, H=2, K=128, V=128, seed=612, gate="g", h0=True, dht=True),
]

SIMPLE_KEYS = ("q", "k", "v", "g", "g_gamma", "h0", "dht", "do")


def simple_inputs(c):
    rng = np.random.default_rng(c["seed"])
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    q = rng.standard_normal((B, T, H, K), dtype=np.float32)
    k = rng.standard_normal((B, T, H, K), dtype=np.float32)
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    g = logsigmoid(rng.standard_normal((B, T, H)).astype(np.float32)).astype(np.float32) \
        if c["gate"] in ("g", "both") else None
    g_gamma = (-np.abs(rng.random(H, dtype=np.float32)) * 0.5).astype(np.float32) \
        if c["gate"] in ("gamma", "both") else None
    cu = c.get("cu")
    N = len(cu) - 1 if cu else B
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("h0") else None
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32) if c.get("dht") else None
    return dict(q=q, k=k, v=v, g=g, g_gamma=g_gamma, h0=h0, dht=dht, do=do, cu=cu, C=c.get("C", 64),
                scale=c.get("scale", K ** -0.5))


def load(name):
    c = next(x for x in SIMPLE_CASES if x["name"] == name)
    inp = simple_inputs(c)
    fx = dict(np.load(GOLDEN_DIR / f"simple_{name}.npz"))
    want = str(fx.pop("input_digest"))
    got = digest(*[inp[k] for k in SIMPLE_KEYS])
    if want != got:
        raise RuntimeError(f"golden inputs for simple/{name} drifted: {got} != {want}")
    return c, inp, fx


def pad_decay(inp):
    """The reference's Torch code pads each sequence to a multiple of the chunk size and
    keeps g_gamma on the padded steps (tests/src/ops/simple_gla/chunk.py:72-137,
    :383-395), so its final state carries exp(g_gamma * pad) of extra decay when the
    length is ragged (its JAX operator asserts T % chunk_size == 0 instead,
    tops/ops/simple_gla/chunk.py:493).  Returns that factor [N, H, 1, 1]."""
    B, T, H, K = inp["q"].shape
    C = inp["C"]
    lens = np.diff(inp["cu"]) if inp["cu"] else np.full(B, T)
    pad = (-lens) % C
    if inp["g_gamma"] is None:
        return np.ones((len(lens), H, 1, 1))
    return np.exp(pad[:, None].astype(np.float64) * inp["g_gamma"][None, :].astype(np.float64))[..., None, None]
