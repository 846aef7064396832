"""Tensor-core (tcgen05) grouped GEMM path vs the oracle and vs the
CUDA-core path, through the C ABI.  Collected after test_gpu_layer.py so the
routing, decode and CUDA-core checks report first."""
import numpy as np
import pytest

from conftest import GOLDEN
from test_gpu_layer import L, bf16_to_f32, check_layer_fixture, engine  # noqa: F401

pytestmark = pytest.mark.gpu
LAYER_FIXTURES = sorted(p.name for p in GOLDEN.glob("layer_*.npz"))


@pytest.mark.parametrize("name", LAYER_FIXTURES)
def test_layer_matches_reference_tcgen05(name, engine, synth, L):
    check_layer_fixture(name, 0, engine, synth, L)


def test_tensor_core_path_matches_simt_path(engine, synth, L):
    shape = synth.small_shape(hidden=256, intermediate=320, experts=8, top_k=3, tokens=200)
    li = synth.make_layer(shape, seed=31)
    engine.upload_layer(li)
    res = {}
    for path in (L.GEMM_SIMT, L.GEMM_TCGEN05):
        out = engine.forward_host(L.Engine.cfg(shape, gemm_path=path), li.x)
        P = 200 * 3
        res[path] = dict(out=out, h=engine.read(L.BUF_HPERM, (P, 320), np.uint16),
                         y=engine.read(L.BUF_YPERM, (P, 256), np.float32))
    hs = bf16_to_f32(res[L.GEMM_SIMT]["h"])
    ht = bf16_to_f32(res[L.GEMM_TCGEN05]["h"])
    # same products, different fp32 summation order, then bf16 rounding
    assert np.allclose(ht, hs, rtol=2 ** -7, atol=1e-4), np.abs(ht - hs).max()
    ys, yt = res[L.GEMM_SIMT]["y"], res[L.GEMM_TCGEN05]["y"]
    assert np.allclose(yt, ys, rtol=1e-3, atol=1e-4), np.abs(yt - ys).max()


