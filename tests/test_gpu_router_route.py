"""The decode-sized router and permutation as one launch against two.

For batches whose router fits one block's shared memory (E <= 64) and whose
assignments fit the single-block permutation, the router kernel's last block
runs the permutation (router_route_kernel); MOE_B200_FUSED_ROUTE=0 at engine
creation launches the router and route_small_kernel separately.  The same
top-k code and the same stable counting sort produce the same bytes, so every
output agrees bit for bit, with one launch fewer.  The cases cover one token,
a shared expert, a skewed routing with experts nobody picked, and several
router blocks whose ids the last one reads.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


def engine_with_fusion(L, on):
    old = os.environ.get("MOE_B200_FUSED_ROUTE")
    os.environ["MOE_B200_FUSED_ROUTE"] = "1" if on else "0"
    try:
        return L.Engine(0)
    finally:
        if old is None:
            del os.environ["MOE_B200_FUSED_ROUTE"]
        else:
            os.environ["MOE_B200_FUSED_ROUTE"] = old


@pytest.mark.parametrize("hidden,inter,experts,top_k,tokens,shared,skew", [
    (1024, 512, 32, 4, 1, False, None),          # one token, one router block
    (1024, 512, 32, 4, 256, True, None),         # 128 router blocks, shared expert
    (2880, 256, 32, 4, 96, False, "zipf1.1"),    # skewed: some experts get no rows
    (512, 256, 64, 8, 40, True, None),           # 64 experts, top-8
], ids=["t1", "t256_shared", "skewed", "e64"])
def test_fused_router_route_matches_two_launches(L, synth, hidden, inter, experts, top_k, tokens, shared, skew):
    shape = synth.small_shape(name="rr", hidden=hidden, intermediate=inter, experts=experts, top_k=top_k,
                              tokens=tokens, shared=shared, skew=skew)
    li = synth.make_layer(shape, seed=hidden + experts + tokens)
    outs, launches = [], []
    for on in (True, False):
        eng = engine_with_fusion(L, on)
        try:
            eng.upload_layer(li, layer=0)
            for _ in range(2):   # the second call reuses the counter the first left at 0
                out = eng.forward_host(L.Engine.cfg(shape), li.x)
            outs.append(out)
            launches.append(eng.launches())
        finally:
            eng.close()
    a, b = outs
    for k in ("ids", "w", "perm", "y_f32", "y_bf16"):
        assert np.array_equal(np.asarray(a[k]).view(np.uint8), np.asarray(b[k]).view(np.uint8)), k
    assert launches[0] == launches[1] - 1, launches
