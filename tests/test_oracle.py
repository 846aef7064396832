"""Pins the CPU oracle (oracle/moe_oracle.c) to the reference.

Against the golden fixtures written by tests/golden/make_golden.py from the
reference's own compiled hot path, and -- where the reference library was
built in this checkout -- against that library on fresh seeds.  Everything
here is bit-exact: ids, weights, scores and layer outputs compare as bit
patterns.
"""
import numpy as np
import pytest

from conftest import GOLDEN, block_from_golden, golden, layer_from_golden

LAYER_FIXTURES = sorted(p.name for p in GOLDEN.glob("layer_*.npz"))
BLOCK_FIXTURES = sorted(p.name for p in GOLDEN.glob("block_*.npz") if p.name != "block_tables.npz")


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_decode_tables(port):
    g = golden("decode_tables.npz")
    e8m0 = np.array([port.lib.mo_e8m0_to_f32(v) for v in range(256)], np.float32)
    e2m1 = np.array([port.lib.mo_mxfp4_value(c) for c in range(16)], np.float32)
    assert np.array_equal(bits(e8m0), bits(g["e8m0"]))
    assert np.array_equal(bits(e2m1), bits(g["e2m1"]))
    # known answers from the reference source itself
    assert e8m0[127] == 1.0 and e8m0[0] == 2.0 ** -127 and np.isinf(e8m0[255])
    assert list(e2m1[:8]) == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    silu = np.array([port.lib.mo_silu(float(v)) for v in g["silu_x"]], np.float32)
    assert np.array_equal(bits(silu), bits(g["silu_y"]))


@pytest.mark.parametrize("name", LAYER_FIXTURES)
def test_layer_matches_reference_fixture(name, port, synth):
    g = golden(name)
    li = layer_from_golden(synth, g)
    y, ids, w, ties = port.moe_layer(li)
    assert ties == 0
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(bits(w), bits(g["w"]))
    assert np.array_equal(bits(y), bits(g["y"]))
    _, _, scores, _ = port.router_topk(li)
    assert np.array_equal(bits(scores), bits(g["scores"]))


def test_sigmoid_router_fixture(port, synth):
    g = golden("router_sigmoid.npz")
    shape = synth.small_shape(top_k=int(g["top_k"]), experts=int(g["experts"]), hidden=int(g["hidden"]),
                              tokens=g["x"].shape[0])
    li = synth.LayerInputs(shape, g["router"], None, None, None, g["x"])
    ids, w, scores, ties = port.router_topk(li, score_sigmoid=1, norm_topk=int(g["norm_topk"]),
                                            routed_scale=float(g["routed_scale"]))
    assert ties == 0
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(bits(w), bits(g["w"]))
    assert np.array_equal(bits(scores), bits(g["scores"]))


@pytest.mark.parametrize("name", ["router_group_limit.npz", "router_group_limit_e1.npz",
                                  "router_group_limit_uneven.npz", "router_group_limit_all.npz"])
def test_group_limit_router_fixture(port, synth, name):
    """Sigmoid router with a DeepSeek-style group limit, against the compiled
    reference's own output (generation_router.cpp.inc:484-558)."""
    g = golden(name)
    shape = synth.small_shape(top_k=int(g["top_k"]), experts=int(g["experts"]), hidden=int(g["hidden"]),
                              tokens=g["x"].shape[0])
    li = synth.LayerInputs(shape, g["router"], None, None, None, g["x"])
    ids, w, scores, ties = port.router_topk(li, score_sigmoid=1, norm_topk=int(g["norm_topk"]),
                                            routed_scale=float(g["routed_scale"]), n_group=int(g["n_group"]),
                                            topk_group=int(g["topk_group"]))
    assert ties == 0
    assert np.array_equal(bits(scores), bits(g["scores"]))
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(bits(w), bits(g["w"]))


def test_grouping_fixture(port):
    g = golden("grouping.npz")
    ok, out, batches, cnt = port.group_tokens(g["token"], g["expert"], g["score"], g["layer"])
    assert ok == int(g["ok"])
    sorted_ = np.array([(a.token_index, a.layer, a.expert) for a in out], np.uint32)
    assert np.array_equal(sorted_, g["sorted"])
    b = np.array([(x.layer, x.expert, x.first_sorted_index, x.token_count) for x in batches[:cnt]], np.uint32)
    assert np.array_equal(b, g["batches"])


def test_grouping_edge_cases(port):
    # empty input fails with zero batches; one assignment is one batch
    # (token_grouping.cpp.inc:9-28)
    ok, _, _, cnt = port.group_tokens([], [])
    assert ok == 0 and cnt == 0
    ok, out, batches, cnt = port.group_tokens([5], [3])
    assert ok == 1 and cnt == 1 and batches[0].token_count == 1 and batches[0].expert == 3


def test_tail_block_dot(port, synth):
    rng = np.random.default_rng(5)
    for cols in (1, 17, 31, 33, 80, 100):
        pk = synth.gen_mxfp4(rng, (), 4, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        out = port.mxfp4_dot_rows(pk, x)
        # exact rational value, independent of the summation order
        vals = np.zeros((4, cols), np.float64)
        nblk = (cols + 31) // 32
        for r in range(4):
            for b in range(nblk):
                blk = pk[r, b * 17:(b + 1) * 17]
                s = 2.0 ** (int(blk[0]) - 127)
                for i in range(min(32, cols - b * 32)):
                    code = (blk[1 + i] & 15) if i < 16 else (blk[1 + i - 16] >> 4)
                    vals[r, b * 32 + i] = port.lib.mo_mxfp4_value(int(code)) * s
        want = vals @ x.astype(np.float64)
        assert np.allclose(out, want, rtol=1e-5, atol=1e-6)


@pytest.fixture(scope="module")
def ref_lib(oracle_mod):
    if not oracle_mod.REF_SO.exists():
        if not oracle_mod.REFERENCE_ROOT.is_dir():
            pytest.skip("reference sources absent; fixtures pin the oracle instead")
        oracle_mod.build(ref=True)
    return oracle_mod


@pytest.mark.parametrize("seed", [21, 22])
def test_port_matches_reference_fresh_seeds(seed, ref_lib, port, synth):
    for shape in (synth.small_shape(tokens=12, experts=12, top_k=3),
                  synth.small_shape(name="s2", hidden=96, intermediate=64, tokens=9, shared=True)):
        li = synth.make_layer(shape, seed=seed)
        ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
        try:
            y2, i2, w2 = ref.moe_layer(li)
        finally:
            ref.close()
        y1, i1, w1, ties = port.moe_layer(li)
        assert ties == 0
        assert np.array_equal(i1, i2)
        assert np.array_equal(bits(w1), bits(w2))
        assert np.array_equal(bits(y1), bits(y2))


def test_block_fixtures_exist():
    assert BLOCK_FIXTURES == ["block_gelu_erf.npz", "block_gemma.npz", "block_router_scalar.npz",
                              "block_router_scale.npz", "block_silu_vector.npz"]


@pytest.mark.parametrize("name", BLOCK_FIXTURES)
def test_block_matches_reference_fixture(name, port, synth, oracle_mod):
    """Gemma-style MoE blocks -- activation, RMSNorms around the experts,
    down scales, shared-expert gate -- against the compiled reference's own
    composition of them (generation_mlp.cpp.inc:776-1442)."""
    g = golden(name)
    li = layer_from_golden(synth, g)
    blk, hidden = block_from_golden(oracle_mod, g)
    y, ids, w, ties = port.moe_block(li, blk, hidden=hidden)
    assert ties == 0
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(bits(w), bits(g["w"]))
    assert np.array_equal(bits(y), bits(g["y"]))
    # the options took effect: the plain layer gives a different output
    y_plain, _, _, _ = port.moe_layer(li)
    assert not np.array_equal(bits(y), bits(y_plain))


def test_block_needs_hidden_for_the_routed_pre_norm(port, synth, oracle_mod):
    g = golden("block_gemma.npz")
    li = layer_from_golden(synth, g)
    blk, _ = block_from_golden(oracle_mod, g)
    with pytest.raises(RuntimeError):
        port.moe_block(li, blk, hidden=None)


def test_block_tables(port, oracle_mod):
    """GELU (erf and tanh forms), SiLU and RMSNorm (plain and Gemma unit
    offset) against the reference's own functions."""
    g = golden("block_tables.npz")
    for mode in (0, 1, 2):
        got = np.array([port.lib.mo_gated_activation(mode, float(a), float(u))
                        for a, u in zip(g["act_x"], g["act_up"])], np.float32)
        assert np.array_equal(bits(got), bits(g[f"act{mode}"])), mode
    P = lambda a: a.ctypes.data_as(oracle_mod._f32p)
    for i in range(3):
        v, w = g[f"norm{i}_in"], g[f"norm{i}_w"]
        for tag, unit in (("plain", 0), ("unit", 1)):
            out = np.zeros_like(v)
            assert port.lib.mo_rmsnorm(P(v), P(w), v.size, 1e-6, unit, P(out))
            assert np.array_equal(bits(out), bits(g[f"norm{i}_{tag}"])), (i, tag)


@pytest.mark.parametrize("seed", [41, 42])
def test_port_matches_reference_block_fresh_seeds(seed, ref_lib, port, synth):
    """Fresh seeds through both: every option on, with and without the shared
    expert, one ragged shape."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    opts = dict(activation=seed % 3, unit_offset=bool(seed % 2), pre_norm2=True, post_norm1=True,
                post_norm2=True, post_norm=True, down_scale="element", shared_gate_inp=True,
                router_scale="element" if seed % 2 else "scalar")
    for shape in (synth.small_shape(name="f1", shared=True, tokens=6, experts=8, top_k=2),
                  synth.small_shape(name="f2", hidden=80, intermediate=100, tokens=5, experts=8, top_k=3)):
        li = synth.make_layer(shape, seed=seed)
        blk, hidden = mg.block_inputs(shape, seed, opts)
        ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk, block=blk))
        try:
            y2, i2, w2 = ref.moe_block(li, blk, hidden=hidden)
        finally:
            ref.close()
        y1, i1, w1, ties = port.moe_block(li, blk, hidden=hidden)
        assert ties == 0
        assert np.array_equal(i1, i2)
        assert np.array_equal(bits(w1), bits(w2))
        assert np.array_equal(bits(y1), bits(y2))


EXTREME_SHAPES = {
    # one 8-element partial block per row, a one-row intermediate
    "h8_i1": dict(hidden=8, intermediate=1, experts=4, top_k=2, tokens=5),
    # a single expert (softmax over one score), with the shared expert
    "e1_shared": dict(hidden=40, intermediate=33, experts=1, top_k=1, tokens=3, shared=True),
    # every expert selected, renormalised
    "k_eq_e": dict(hidden=64, intermediate=32, experts=6, top_k=6, tokens=4, norm_topk=True),
    # one token, 32 of 40 experts (the largest k), ragged blocks on both sides
    "t1_k32": dict(hidden=72, intermediate=40, experts=40, top_k=32, tokens=1),
}


@pytest.mark.parametrize("name", sorted(EXTREME_SHAPES))
def test_port_matches_reference_extreme_shapes(name, ref_lib, port, synth):
    """The oracle the GPU tests compare against, pinned to the compiled
    reference where shapes are at their limits: partial 32-element blocks,
    one intermediate row, one expert, k = E, k = 32, one token."""
    shape = synth.small_shape(name=name, **EXTREME_SHAPES[name])
    li = synth.make_layer(shape, seed=51)
    ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
    try:
        y2, i2, w2 = ref.moe_layer(li)
        _, _, s2 = ref.router_topk(li)
    finally:
        ref.close()
    y1, i1, w1, ties = port.moe_layer(li)
    _, _, s1, _ = port.router_topk(li)
    assert ties == 0
    assert np.array_equal(bits(s1), bits(s2))
    assert np.array_equal(i1, i2)
    assert np.array_equal(bits(w1), bits(w2))
    assert np.array_equal(bits(y1), bits(y2))


def test_oracle_struct_layout(oracle_mod, tmp_path):
    """The ctypes mirror of mo_layer_t has the C header's size and field
    offsets (compiled with the host C compiler)."""
    import ctypes
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    inc = oracle_mod.HERE
    L = oracle_mod.MoLayer
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "moe_oracle.h"', "int main(void) {",
             'printf("size %zu\\n", sizeof(mo_layer_t));']
    for fname, _ in L._fields_:
        lines.append(f'printf("{fname} %zu\\n", offsetof(mo_layer_t, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(inc), str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.split("\n") if l)
    assert int(got["size"]) == ctypes.sizeof(L)
    for fname, _ in L._fields_:
        assert int(got[fname]) == getattr(L, fname).offset, fname


LAYER_FUNCTION_SHAPES = {
    "e12_k3": dict(tokens=12, experts=12, top_k=3),
    "shared": dict(name="s2", hidden=96, intermediate=64, tokens=9, shared=True),
    "norm_topk": dict(name="nt", hidden=64, intermediate=48, experts=8, top_k=4, tokens=6, norm_topk=True),
    # config 4's hidden and intermediate sizes with the shared expert, 12 experts, top-8
    "c4_dims": dict(name="c4d", hidden=7168, intermediate=2048, experts=12, top_k=8, tokens=2, shared=True),
    **EXTREME_SHAPES,
}


@pytest.mark.parametrize("name", sorted(LAYER_FUNCTION_SHAPES))
def test_reference_layer_function_matches_composed_layer(name, ref_lib, port, synth, tmp_path):
    """The reference's moe_layer_moe_mlp_f32 itself -- its experts found as
    tensor records over a shard file, mapped and decoded by the engine's own
    record path -- against the leaf composition (ref_moe_layer) and the
    oracle restatement, bit for bit."""
    shape = synth.small_shape(name=name, **{k: v for k, v in LAYER_FUNCTION_SHAPES[name].items() if k != "name"})
    li = synth.make_layer(shape, seed=61)
    ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
    try:
        y_fn, i_fn, w_fn = ref.moe_layer_engine(li, tmp_path / "shard.bin")
        y_c, i_c, w_c = ref.moe_layer(li)
    finally:
        ref.close()
    assert np.array_equal(i_fn, i_c)
    assert np.array_equal(bits(w_fn), bits(w_c))
    assert np.array_equal(bits(y_fn), bits(y_c))
    y_p, i_p, w_p, ties = port.moe_layer(li)
    assert ties == 0
    assert np.array_equal(i_fn, i_p)
    assert np.array_equal(bits(w_fn), bits(w_p))
    assert np.array_equal(bits(y_fn), bits(y_p))


BLOCK_FUNCTION_OPTIONS = {
    "all_on": dict(activation=1, unit_offset=True, pre_norm2=True, post_norm1=True, post_norm2=True, post_norm=True,
                   down_scale="element", shared_gate_inp=True, router_scale="element"),
    "tanh_scalar": dict(activation=2, unit_offset=False, pre_norm2=True, post_norm1=False, post_norm2=True,
                        post_norm=True, down_scale="expert", shared_gate_inp=False, router_scale="scalar"),
    "silu_post_only": dict(activation=0, unit_offset=False, pre_norm2=False, post_norm1=True, post_norm2=False,
                           post_norm=False, down_scale="scalar", shared_gate_inp=True, router_scale=None),
}


@pytest.mark.parametrize("opt", sorted(BLOCK_FUNCTION_OPTIONS))
def test_reference_layer_function_matches_composed_block(opt, ref_lib, port, synth, tmp_path):
    """moe_layer_moe_mlp_f32 itself with Gemma-style block parts (pre-norm,
    post-FFW norms, down scales, shared-expert gate, router input scale)
    against the leaf composition (ref_moe_block) and the restatement."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    opts = BLOCK_FUNCTION_OPTIONS[opt]
    for shape in (synth.small_shape(name="bf1", shared=True, tokens=6, experts=8, top_k=2),
                  synth.small_shape(name="bf2", hidden=80, intermediate=100, tokens=5, experts=8, top_k=3)):
        li = synth.make_layer(shape, seed=71)
        blk, hidden = mg.block_inputs(shape, 71, opts)
        ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk, block=blk))
        try:
            y_fn, i_fn, w_fn = ref.moe_block(li, blk, hidden=hidden, shard_path=tmp_path / "shard.bin")
            y_c, i_c, w_c = ref.moe_block(li, blk, hidden=hidden)
        finally:
            ref.close()
        assert np.array_equal(i_fn, i_c), shape.name
        assert np.array_equal(bits(w_fn), bits(w_c)), shape.name
        assert np.array_equal(bits(y_fn), bits(y_c)), shape.name
        y_p, i_p, w_p, ties = port.moe_block(li, blk, hidden=hidden)
        assert ties == 0
        assert np.array_equal(bits(y_fn), bits(y_p)), shape.name


ROUTER_FUNCTION_CASES = {
    # sigmoid scores with a routed scale, renormalised
    "sigmoid_scaled": dict(shape=dict(hidden=96, intermediate=64, experts=16, top_k=4, tokens=7, norm_topk=True),
                           route=dict(sigmoid=True, routed_scale=2.5)),
    # sigmoid with the group limit: 8 groups of 4 experts, 3 kept
    "group_limit": dict(shape=dict(hidden=64, intermediate=48, experts=32, top_k=6, tokens=6, shared=True),
                        route=dict(sigmoid=True, routed_scale=1.0, n_group=8, topk_group=3)),
    # sigmoid, not renormalised, one expert per group, 5 groups kept
    "group_of_one": dict(shape=dict(hidden=80, intermediate=40, experts=16, top_k=4, tokens=5),
                         route=dict(sigmoid=True, routed_scale=1.5, n_group=16, topk_group=5)),
}


@pytest.mark.parametrize("case", sorted(ROUTER_FUNCTION_CASES))
def test_reference_layer_function_matches_sigmoid_group_routing(case, ref_lib, port, synth, tmp_path):
    """DeepSeek-style routing (sigmoid scores, routed scale, group limit)
    through moe_layer_moe_mlp_f32 itself, against the composition and the
    restatement, bit for bit."""
    c = ROUTER_FUNCTION_CASES[case]
    shape = synth.small_shape(name=case, **c["shape"])
    r = c["route"]
    li = synth.make_layer(shape, seed=81)
    ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=shape.norm_topk, **r))
    try:
        y_fn, i_fn, w_fn = ref.moe_layer_engine(li, tmp_path / "shard.bin")
        y_c, i_c, w_c = ref.moe_layer(li)
    finally:
        ref.close()
    assert np.array_equal(i_fn, i_c)
    assert np.array_equal(bits(w_fn), bits(w_c))
    assert np.array_equal(bits(y_fn), bits(y_c))
    y_p, i_p, w_p, ties = port.moe_layer(li, score_sigmoid=int(r["sigmoid"]), routed_scale=r["routed_scale"],
                                         n_group=r.get("n_group", 0), topk_group=r.get("topk_group", 0))
    assert ties == 0
    assert np.array_equal(i_fn, i_p)
    assert np.array_equal(bits(w_fn), bits(w_p))
    assert np.array_equal(bits(y_fn), bits(y_p))


@pytest.mark.parametrize("norm_topk", [False, True], ids=["no_renorm", "renorm"])
@pytest.mark.parametrize("shared_missing", [False, True], ids=["shared_present", "shared_missing"])
def test_reference_partial_failure_matches_port(norm_topk, shared_missing, ref_lib, port, synth, tmp_path):
    """The reference's partial-failure policy through its own layer function
    (generation_mlp.cpp.inc:1219-1282): experts without records drop out of
    the sum, a renormalising router divides the others' combine weights by
    their sum, and the router's ids and weights stay as routed.  Held bit for
    bit to the restatement given the same missing experts."""
    shape = synth.small_shape(name="pf", hidden=96, intermediate=64, experts=8, top_k=3, tokens=24, shared=True,
                              norm_topk=norm_topk)
    li = synth.make_layer(shape, seed=91)
    present = np.ones(shape.experts + 1, np.uint8)
    present[[2, 5]] = 0
    if shared_missing:
        present[shape.experts] = 0
    ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k, norm_topk=norm_topk))
    try:
        y_fn, i_fn, w_fn = ref.moe_layer_engine(li, tmp_path / "shard.bin", present=present)
    finally:
        ref.close()
    y_p, i_p, w_p, ties = port.moe_layer(li, present=present)
    assert ties == 0
    assert np.isin(i_p, [2, 5]).any()     # some token routes to a missing expert
    assert np.array_equal(i_fn, i_p)
    assert np.array_equal(bits(w_fn), bits(w_p))
    assert np.array_equal(bits(y_fn), bits(y_p))
    # Leaving the missing experts' terms at zero with the routed weights (their
    # down weights zeroed) is the policy without renormalisation only.
    zeroed = synth.LayerInputs(shape, li.router, li.gate, li.up, li.down.copy(), li.x, li.shared_gate, li.shared_up,
                               np.zeros_like(li.shared_down) if shared_missing else li.shared_down)
    zeroed.down[[2, 5]] = 0
    y_z, _, _, _ = port.moe_layer(zeroed)
    assert np.array_equal(y_z, y_p) != norm_topk


def test_reference_fails_a_token_whose_experts_are_all_missing(ref_lib, port, synth, tmp_path):
    """The reference's layer function fails when none of a token's selected
    experts has records (generation_mlp.cpp.inc:1219-1239); so does the
    restatement."""
    shape = synth.small_shape(name="am", hidden=64, intermediate=48, experts=6, top_k=2, tokens=4)
    li = synth.make_layer(shape, seed=93)
    ids, _, _, _ = port.router_topk(li)
    present = np.ones(shape.experts + 1, np.uint8)
    present[list(ids[0])] = 0
    ref = ref_lib.Ref(ref_lib.metadata_json(shape.top_k))
    try:
        with pytest.raises(RuntimeError):
            ref.moe_layer_engine(li, tmp_path / "shard.bin", present=present)
    finally:
        ref.close()
    with pytest.raises(RuntimeError):
        port.moe_layer(li, present=present)
