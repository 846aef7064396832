"""Host-buffer calls on large batches (moe_b200_layer_forward_host without
the permutation output) copy x in token chunks, route each chunk as it lands,
and combine and copy back chunk by chunk.  Every token's result must be the
one the unchunked call computes, bit for bit: outputs, ids and weights, with
and without the shared expert, with the block combine parts (post-norms,
down scales, shared-expert gate), and for batch sizes that leave a short last
chunk."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


def same(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


@pytest.mark.parametrize("tokens,shared,block", [
    (4096, True, False),   # eight equal chunks
    (5003, True, False),   # a short last chunk
    (4500, False, False),  # no shared expert
    (4200, True, True),    # block combine parts and the shared-expert gate
], ids=["even", "ragged", "no_shared", "block"])
def test_chunked_host_call_matches_unchunked(L, synth, tokens, shared, block):
    shape = synth.small_shape(name="pipe", hidden=256, intermediate=192, experts=8, top_k=2, tokens=tokens,
                              shared=shared)
    li = synth.make_layer(shape, seed=tokens)
    eng = L.Engine(0)
    try:
        eng.upload_layer(li, layer=0)
        if block:
            rng = np.random.default_rng(3)
            H = shape.hidden
            eng.upload_block(0, post_norm1=rng.normal(0, 0.2, H), post_norm2=rng.normal(0, 0.2, H),
                             post_norm=rng.normal(0, 0.2, H), down_scale=rng.uniform(0.5, 1.5, shape.experts),
                             shared_gate_inp=li.router[:1].copy())
        cfg = L.Engine.cfg(shape)
        ref = eng.forward_host(cfg, li.x, want_perm=True)    # the permutation output: one piece
        got = eng.forward_host(cfg, li.x, want_perm=False)   # chunked
        again = eng.forward_host(cfg, li.x, want_perm=False)
    finally:
        eng.close()
    for k in ("y_bf16", "y_f32", "ids", "w"):
        assert same(got[k], ref[k]), k
        assert same(again[k], ref[k]), k
    assert np.abs(ref["y_f32"]).max() > 0
