"""Tensor-core (tcgen05) grouped GEMM path vs the oracle and vs the
CUDA-core path, through the C ABI.  Collected after test_gpu_layer.py so the
routing, decode and CUDA-core checks report first."""
import numpy as np
import pytest

from conftest import GOLDEN
from test_gpu_layer import MAX_ABS, MEAN_REL, L, bf16_to_f32, check_layer_fixture, engine, errors  # noqa: F401

pytestmark = pytest.mark.gpu
LAYER_FIXTURES = sorted(p.name for p in GOLDEN.glob("layer_*.npz"))


@pytest.mark.parametrize("path", [0, 2], ids=["blockscaled", "tmem_decode"])
@pytest.mark.parametrize("name", LAYER_FIXTURES)
def test_layer_matches_reference_tcgen05(name, path, engine, synth, L):
    check_layer_fixture(name, path, engine, synth, L)


def test_tensor_core_path_matches_simt_path(engine, synth, L):
    shape = synth.small_shape(hidden=256, intermediate=320, experts=8, top_k=3, tokens=200)
    li = synth.make_layer(shape, seed=31)
    engine.upload_layer(li)
    res = {}
    for path in (L.GEMM_SIMT, L.GEMM_TMEM_DECODE):
        out = engine.forward_host(L.Engine.cfg(shape, gemm_path=path), li.x)
        P = 200 * 3
        res[path] = dict(out=out, h=engine.read(L.BUF_HPERM, (P, 320), np.uint16),
                         y=engine.read(L.BUF_YPERM, (P, 256), np.float32))
    hs = bf16_to_f32(res[L.GEMM_SIMT]["h"])
    ht = bf16_to_f32(res[L.GEMM_TMEM_DECODE]["h"])
    # same products, different fp32 summation order, then bf16 rounding
    assert np.allclose(ht, hs, rtol=2 ** -7, atol=1e-4), np.abs(ht - hs).max()
    ys, yt = res[L.GEMM_SIMT]["y"], res[L.GEMM_TMEM_DECODE]["y"]
    assert np.allclose(yt, ys, rtol=1e-3, atol=1e-4), np.abs(yt - ys).max()


def jitter_all_scales(synth, li, seed, spread=4, up=1):
    rng = np.random.default_rng(seed)
    for name in ("gate", "up", "down", "shared_gate", "shared_up", "shared_down"):
        a = getattr(li, name, None)
        if a is not None:
            setattr(li, name, synth.jitter_scales(a, rng, spread, up))


@pytest.mark.parametrize("jitter", [False, True], ids=["one_scale", "varied_scales"])
@pytest.mark.parametrize("tokens,top_k,experts", [(200, 3, 8), (40, 2, 16), (700, 4, 8)])
def test_blockscaled_expert_outputs_match_simt(engine, synth, L, tokens, top_k, experts, jitter):
    """Per permuted row, the block-scaled GEMMs' fp32 expert outputs against
    the CUDA-core path (same products; the intermediate is rounded as two
    E4M3 terms instead of bf16, so the bar is a relative one).  The varied
    case gives every 32-element weight block its own scale, which pins the
    placement of the weight scale factors in tensor memory row by row."""
    shape = synth.small_shape(hidden=256, intermediate=320, experts=experts, top_k=top_k, tokens=tokens)
    li = synth.make_layer(shape, seed=41 + tokens)
    if jitter:
        jitter_all_scales(synth, li, seed=tokens)
    engine.upload_layer(li)
    P, H = tokens * top_k, 256
    out_s = engine.forward_host(L.Engine.cfg(shape, gemm_path=L.GEMM_SIMT), li.x)
    ys = engine.read(L.BUF_YPERM, (P, H), np.float32)
    out_b = engine.forward_host(L.Engine.cfg(shape, gemm_path=L.GEMM_BLOCKSCALED), li.x)
    yb = engine.read(L.BUF_YPERM, (P, H), np.float32)
    assert np.array_equal(out_s["ids"], out_b["ids"])
    scale = np.abs(ys).mean()
    assert np.abs(yb - ys).max() <= 0.05 * np.abs(ys).max() + 1e-6, np.abs(yb - ys).max()
    assert np.abs(yb - ys).mean() <= 5e-3 * scale, (np.abs(yb - ys).mean(), scale)




@pytest.mark.parametrize("path", [0, 1, 2], ids=["blockscaled", "simt", "tmem_decode"])
@pytest.mark.parametrize("tokens,top_k,experts,shared", [(40, 2, 8, False), (200, 3, 8, True)])
def test_varied_weight_scales_match_oracle(engine, synth, L, port, path, tokens, top_k, experts, shared):
    """Layer output with per-block weight scales against the CPU oracle."""
    shape = synth.small_shape(hidden=256, intermediate=320, experts=experts, top_k=top_k, tokens=tokens,
                              shared=shared)
    li = synth.make_layer(shape, seed=77 + tokens)
    jitter_all_scales(synth, li, seed=5 + tokens)
    engine.upload_layer(li)
    out = engine.forward_host(L.Engine.cfg(shape, gemm_path=path), li.x)
    y_ref, ids, _, _ = port.moe_layer(li)
    assert np.array_equal(out["ids"], ids)
    mx, mr = errors(out["y_f32"], y_ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
