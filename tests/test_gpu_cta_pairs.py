"""CTA-pair GEMMs (cta_group::2) against the one-CTA GEMMs and the oracle.

The 128-token tiles of the exact block-scaled path run on CTA pairs: one
M = 256 MMA over the two SMs of a TPC, each CTA holding its 128 weight rows
and half of the tile's token rows.  MOE_B200_CTA_PAIRS=0 at engine creation
selects the one-CTA kernels.  Both compute each output element from the same
products accumulated in the same K order, so their outputs agree bit for bit;
one case is also held to the oracle at the layer bars.  The cases cover
paired gate/up and down, an odd number of intermediate row tiles (gate/up
falls back to one CTA, down pairs), an odd number of hidden row tiles (the
reverse), ragged group tails down to a single token, and a skewed routing.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-2


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


def engine_with_pairs(L, on, **kw):
    old = os.environ.get("MOE_B200_CTA_PAIRS")
    os.environ["MOE_B200_CTA_PAIRS"] = "1" if on else "0"
    try:
        return L.Engine(0, **kw)
    finally:
        if old is None:
            del os.environ["MOE_B200_CTA_PAIRS"]
        else:
            os.environ["MOE_B200_CTA_PAIRS"] = old


def run_both(L, synth, shape, seed):
    li = synth.make_layer(shape, seed=seed)
    rng = np.random.default_rng(seed)
    li.gate = synth.jitter_scales(li.gate, rng, 6, 3)
    li.down = synth.jitter_scales(li.down, rng, 6, 3)
    outs = []
    for on in (True, False):
        eng = engine_with_pairs(L, on)
        try:
            eng.upload_layer(li, layer=0)
            outs.append(eng.forward_host(L.Engine.cfg(shape), li.x))
        finally:
            eng.close()
    return li, outs[0], outs[1]


@pytest.mark.parametrize("hidden,inter,experts,top_k,tokens,shared,skew", [
    (1024, 512, 8, 2, 1200, True, None),       # both GEMMs paired
    (1024, 384, 8, 2, 1200, False, None),      # 3 intermediate row tiles: gate/up one CTA, down paired
    (896, 512, 16, 4, 800, True, None),        # 7 hidden row tiles: gate/up paired, down one CTA
    (1024, 512, 16, 4, 1100, True, "zipf1.1"),  # skewed: tails of 1-10 tokens, 16-column MMAs
], ids=["paired", "odd_inter", "odd_hidden", "skewed"])
def test_pairs_match_single_cta(L, synth, hidden, inter, experts, top_k, tokens, shared, skew):
    shape = synth.small_shape(name="pairs", hidden=hidden, intermediate=inter, experts=experts, top_k=top_k,
                              tokens=tokens, shared=shared, skew=skew)
    li, a, b = run_both(L, synth, shape, seed=hidden + inter + experts)
    # the tiles are 128 tokens wide (the groups average more than 160 rows)
    counts = np.bincount(a["ids"].ravel(), minlength=experts)
    assert (tokens * top_k + (tokens if shared else 0)) / (experts + int(shared)) > 160
    if skew:
        tails = counts % 128
        assert ((tails > 0) & (tails < 16)).any()  # tail tiles narrower than one 16-column MMA
    for k in ("ids", "w", "perm", "y_f32", "y_bf16"):
        assert np.array_equal(np.asarray(a[k]).view(np.uint8), np.asarray(b[k]).view(np.uint8)), k


def test_pairs_match_oracle(L, synth, port):
    shape = synth.small_shape(name="pairs_oracle", hidden=1024, intermediate=512, experts=4, top_k=2, tokens=600,
                              shared=True)
    li = synth.make_layer(shape, seed=5)
    eng = engine_with_pairs(L, True)
    try:
        eng.upload_layer(li, layer=0)
        out = eng.forward_host(L.Engine.cfg(shape), li.x)
    finally:
        eng.close()
    y_ref, ids_ref, w_ref, _ = port.moe_layer(li)
    assert np.array_equal(out["ids"], ids_ref)
    assert np.array_equal(np.asarray(out["w"]).view(np.uint32), np.asarray(w_ref, np.float32).view(np.uint32))
    d = np.abs(out["y_f32"].astype(np.float64) - y_ref.astype(np.float64))
    assert d.max() <= MAX_ABS, d.max()
    assert d.mean() / np.abs(y_ref).mean() <= MEAN_REL
