"""Gemma-style block parts on the GPU (moe_b200_upload_block +
moe_b200_block_forward) against fixtures the compiled reference produced:
GELU activations (erf and tanh forms), the MoE pre-norm of the routed input,
post-FFW norms 1, 2 and final, expert down scales (global, per expert, per
element), the shared-expert gate and the router input scale
(generation_mlp.cpp.inc:94-104, 234-250, 380-570;
generation_router.cpp.inc:316-359).

Bars: ids and weights bit-exact (the router reads the pre-normed or scaled
residual stream exactly as the reference computes it); the block output
within max abs 2e-2 and mean rel 1e-2.
"""
import numpy as np
import pytest

from conftest import GOLDEN, block_from_golden, golden, layer_from_golden
from test_gpu_layer import MAX_ABS, MEAN_REL, bits, errors  # noqa: F401

pytestmark = pytest.mark.gpu
BLOCK_FIXTURES = sorted(p.name for p in GOLDEN.glob("block_*.npz") if p.name != "block_tables.npz")


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


@pytest.fixture(scope="module")
def engine(L):
    e = L.Engine(0)
    yield e
    e.close()


def upload_with_block(engine, li, blk):
    engine.upload_layer(li)
    engine.upload_block(0, pre_norm2=blk.pre_norm2, post_norm1=blk.post_norm1, post_norm2=blk.post_norm2,
                        post_norm=blk.post_norm, down_scale=blk.down_scale, shared_gate_inp=blk.shared_gate_inp,
                        router_scale=blk.router_scale)


@pytest.mark.parametrize("path", [0], ids=["blockscaled"])
@pytest.mark.parametrize("name", BLOCK_FIXTURES)
def test_block_matches_reference_fixture(name, path, engine, synth, L, oracle_mod):
    g = golden(name)
    li = layer_from_golden(synth, g)
    blk, hidden = block_from_golden(oracle_mod, g)
    upload_with_block(engine, li, blk)
    cfg = L.Engine.cfg(li.shape, gemm_path=path, activation=blk.activation, norm_unit_offset=blk.unit_offset,
                       norm_eps=blk.eps)
    out = engine.block_forward_host(cfg, li.x, hidden)
    assert np.array_equal(out["ids"], g["ids"])
    assert np.array_equal(bits(out["w"]), bits(g["w"]))
    mx, mr = errors(out["y_f32"], g["y"])
    print(f"{name}: max abs {mx:.3e} mean rel {mr:.3e}")
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    engine.clear_block(0)
    engine.sync()


def test_block_parts_need_the_residual_stream(engine, synth, L, oracle_mod):
    g = golden("block_gemma.npz")
    li = layer_from_golden(synth, g)
    blk, hidden = block_from_golden(oracle_mod, g)
    upload_with_block(engine, li, blk)
    cfg = L.Engine.cfg(li.shape, activation=blk.activation, norm_unit_offset=blk.unit_offset, norm_eps=blk.eps)
    with pytest.raises(L.MoEError, match="residual stream"):
        engine.forward_host(cfg, li.x)  # the plain forward has no hidden input
    with pytest.raises(L.MoEError, match="block-scaled"):
        engine.block_forward_host(L.Engine.cfg(li.shape, gemm_path=L.GEMM_SIMT, activation=blk.activation), li.x,
                                  hidden)
    engine.clear_block(0)
    engine.sync()


@pytest.mark.parametrize("activation", [1, 2], ids=["gelu_erf", "gelu_tanh"])
def test_gelu_activation_matches_oracle(engine, synth, L, port, oracle_mod, activation):
    """A GELU-gated layer with no other block part, at a real hidden size."""
    shape = synth.small_shape(name="gelu", hidden=1024, intermediate=704, experts=8, top_k=2, tokens=48)
    li = synth.make_layer(shape, seed=61)
    engine.upload_layer(li)
    out = engine.forward_host(L.Engine.cfg(shape, activation=activation), li.x)
    y_ref, ids_ref, w_ref, _ = port.moe_block(li, oracle_mod.Block(activation=activation))
    assert np.array_equal(out["ids"], ids_ref)
    mx, mr = errors(out["y_f32"], y_ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
