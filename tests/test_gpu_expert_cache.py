"""Repacked-expert records on the GPU (moe_b200_export_expert /
moe_b200_import_expert, storage.llm_b200/expert_cache.py).

An engine whose experts were installed from a cache file made by another
engine computes the same layer outputs bit for bit as the engine that
repacked them from the GGUF bytes, and exports the same records again.
Records also install from device memory, and the calls refuse what they
cannot serve: a record of the wrong size, an expert that is not resident.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


@pytest.fixture(scope="module")
def ec(pkg):
    import moe_b200.expert_cache as m
    return m


def _sources(li):
    s = li.shape
    src = {e: (li.gate[e], li.up[e], li.down[e]) for e in range(s.experts)}
    if li.shared_gate is not None:
        src[-1] = (li.shared_gate, li.shared_up, li.shared_down)
    return src


@pytest.mark.parametrize("hidden,inter,experts,top_k,tokens,shared", [
    (1024, 512, 8, 2, 1200, True),   # 128-token tiles on CTA pairs, shared expert
    (896, 384, 16, 4, 96, False),    # padded rows and K (H, I not multiples of 128), decode tiles
], ids=["prefill_shared", "padded_decode"])
def test_cached_experts_match_repacked(L, synth, ec, tmp_path, hidden, inter, experts, top_k, tokens, shared):
    shape = synth.small_shape(name="cache", hidden=hidden, intermediate=inter, experts=experts, top_k=top_k,
                              tokens=tokens, shared=shared)
    li = synth.make_layer(shape, seed=hidden + inter)
    src = _sources(li)
    keys = {(0, e): ec.source_key(*b) for e, b in src.items()}
    path = str(tmp_path / "layer0.b200cache")
    a = L.Engine(0)
    try:
        a.upload_layer(li, layer=0)
        out_a = a.forward_host(L.Engine.cfg(shape), li.x)
        assert ec.save_resident(a, path, hidden, inter, keys) == len(src)
        recs_a = {e: a.export_expert(0, e, hidden, inter) for e in src}
    finally:
        a.close()
    cache = ec.CacheFile(path)
    b = L.Engine(0)
    try:
        b.upload_router(0, np.ascontiguousarray(li.router), experts, hidden)
        for e, (g, u, d) in src.items():
            assert ec.make_resident(b, cache, 0, e, g, u, d, hidden, inter) is True
        out_b = b.forward_host(L.Engine.cfg(shape), li.x)
        for e in src:
            assert np.array_equal(b.export_expert(0, e, hidden, inter), recs_a[e]), e
    finally:
        b.close()
    for k in ("ids", "w", "perm", "y_f32", "y_bf16"):
        assert np.array_equal(np.asarray(out_a[k]).view(np.uint8), np.asarray(out_b[k]).view(np.uint8)), k


def test_record_from_device_memory_and_refusals(L, synth, ec):
    import torch
    shape = synth.small_shape(name="cache_dev", hidden=512, intermediate=256, experts=4, top_k=2, tokens=64)
    li = synth.make_layer(shape, seed=11)
    H, I = shape.hidden, shape.intermediate
    a = L.Engine(0)
    try:
        a.upload_layer(li, layer=0)
        out_a = a.forward_host(L.Engine.cfg(shape), li.x)
        recs = [a.export_expert(0, e, H, I) for e in range(shape.experts)]
        with pytest.raises(L.MoEError, match="not resident"):
            a.export_expert(0, -1, H, I)   # no shared expert was uploaded
    finally:
        a.close()
    b = L.Engine(0)
    try:
        b.upload_router(0, np.ascontiguousarray(li.router), shape.experts, H)
        with pytest.raises(L.MoEError, match="bytes"):
            b.import_expert(0, 0, recs[0][:-1], H, I)
        with pytest.raises(L.MoEError, match="does not match"):
            b.import_expert(0, 0, recs[0], H + 128, I)
        for e, rec in enumerate(recs):
            dev = torch.from_numpy(rec).to("cuda:0")
            b.import_expert(0, e, dev, H, I, on_device=True)
        torch.cuda.synchronize()
        out_b = b.forward_host(L.Engine.cfg(shape), li.x)
    finally:
        b.close()
    for k in ("ids", "w", "y_f32", "y_bf16"):
        assert np.array_equal(np.asarray(out_a[k]).view(np.uint8), np.asarray(out_b[k]).view(np.uint8)), k
