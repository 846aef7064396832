"""Writes the golden fixtures under tests/golden/ from the reference itself.

The reference ships no tests, golden vectors or fixtures, so parity is pinned
by running the reference's own CPU hot path (compiled from its sources into
oracle/_ref/libmoe_ref.so by oracle/Makefile) on seeded synthetic inputs and
recording its outputs here.  Run it in a checkout that has the reference
sources (MOE_REFERENCE_ROOT; its default is set in oracle/oracle.py):

    python tests/golden/make_golden.py [name-prefix]

Small cases store every input; full-size cases store the seed and a sha256 of
the regenerated inputs, so a test can prove it regenerated the same bytes.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle  # noqa: E402


def _load_synth():
    spec = importlib.util.spec_from_file_location("moe_b200_synth", ROOT / "storage.llm_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


synth = _load_synth()
OUT = Path(__file__).resolve().parent

# name -> (shape, seed, tokens or None, store_inputs)
LAYER_CASES = {
    "mini": (synth.small_shape(tokens=16), 1, None, True),
    "tail": (synth.small_shape(name="tail", hidden=80, intermediate=100, tokens=20), 3, None, True),
    "shared": (synth.small_shape(name="shared", shared=True, tokens=20), 4, None, True),
    "norm_topk": (synth.small_shape(name="norm_topk", top_k=4, norm_topk=True, tokens=20), 5, None, True),
    "c0": (synth.CONFIGS[0], 0, None, False),
    "c1_t8": (synth.CONFIGS[1], 0, 8, False),
    "c3_t16": (synth.CONFIGS[3], 0, 16, False),
    # decode at one token (the engine's per-token call) and a mid-sweep batch
    "c1_t1": (synth.CONFIGS[1], 0, 1, False),
    "c1_t32": (synth.CONFIGS[1], 0, 32, False),
    # the largest configuration: H=7168, 256 experts, top-8, shared expert
    "c4_t8": (synth.CONFIGS[4], 0, 8, False),
}


def layer_case(name, shape, seed, tokens, store_inputs):
    li = synth.make_layer(shape, seed=seed, tokens=tokens)
    ref = oracle.Ref(oracle.metadata_json(shape.top_k, norm_topk=shape.norm_topk))
    try:
        y, ids, w = ref.moe_layer(li)
        _, _, scores = ref.router_topk(li)
    finally:
        ref.close()
    rec = dict(hidden=shape.hidden, intermediate=shape.intermediate, experts=shape.experts,
               top_k=shape.top_k, tokens=li.x.shape[0], shared=int(shape.shared),
               norm_topk=int(shape.norm_topk), skew=shape.skew or "", seed=seed,
               digest=li.digest(), ids=ids, w=w, y=y, scores=scores)
    if store_inputs:
        rec.update(router=li.router, gate=li.gate, up=li.up, down=li.down, x=li.x)
        if shape.shared:
            rec.update(shared_gate=li.shared_gate, shared_up=li.shared_up, shared_down=li.shared_down)
    np.savez_compressed(OUT / f"layer_{name}.npz", **rec)
    print(f"layer_{name}: T={li.x.shape[0]} digest={rec['digest'][:16]}")


def sigmoid_case():
    shape = synth.small_shape(name="sigmoid", top_k=3, experts=16, tokens=24)
    li = synth.make_layer(shape, seed=7)
    ref = oracle.Ref(oracle.metadata_json(3, norm_topk=True, sigmoid=True, routed_scale=2.5))
    try:
        ids, w, scores = ref.router_topk(li)
    finally:
        ref.close()
    np.savez_compressed(OUT / "router_sigmoid.npz", router=li.router, x=li.x, ids=ids, w=w, scores=scores,
                        hidden=shape.hidden, experts=shape.experts, top_k=3, norm_topk=1, routed_scale=2.5)
    print("router_sigmoid")


# name -> (experts, n_group, topk_group, top_k, seed): DeepSeek-style group
# limits (generation_router.cpp.inc:484-558), one with a single expert per
# group
GROUP_LIMIT_CASES = {
    "router_group_limit": (32, 8, 3, 4, 13),
    "router_group_limit_e1": (16, 16, 5, 3, 14),
    # combinations the reference ignores: groups not dividing the experts,
    # and as many kept groups as groups
    "router_group_limit_uneven": (16, 3, 1, 3, 15),
    "router_group_limit_all": (16, 4, 4, 3, 16),
}


def group_limit_case(name, experts, n_group, topk_group, top_k, seed):
    shape = synth.small_shape(name=name, top_k=top_k, experts=experts, tokens=40)
    li = synth.make_layer(shape, seed=seed)
    ref = oracle.Ref(oracle.metadata_json(top_k, norm_topk=True, sigmoid=True, routed_scale=2.5,
                                          n_group=n_group, topk_group=topk_group))
    try:
        ids, w, scores = ref.router_topk(li)
    finally:
        ref.close()
    np.savez_compressed(OUT / f"{name}.npz", router=li.router, x=li.x, ids=ids, w=w, scores=scores,
                        hidden=shape.hidden, experts=experts, top_k=top_k, norm_topk=1, routed_scale=2.5,
                        n_group=n_group, topk_group=topk_group)
    print(name)


# name -> (shape, seed, options): Gemma-style MoE blocks -- the optional
# activation, norms, down scales and shared-expert gate around the experts
# (generation_mlp.cpp.inc:94-104, 145-175, 234-250, 380-429, 478-570)
BLOCK_CASES = {
    # everything on: GELU (tanh), Gemma norms, routed input from RMSNorm(hidden),
    # per-expert down scale, gated shared expert
    "block_gemma": (synth.small_shape(name="block_gemma", shared=True, top_k=3, experts=12, tokens=16), 31,
                    dict(activation=2, unit_offset=True, eps=1e-6, pre_norm2=True, post_norm1=True,
                         post_norm2=True, post_norm=True, down_scale="expert", shared_gate_inp=True)),
    # GELU (erf), plain norms on the routed outputs only, one global scale
    "block_gelu_erf": (synth.small_shape(name="block_gelu_erf", top_k=2, experts=8, tokens=16), 32,
                       dict(activation=1, eps=1e-5, post_norm2=True, down_scale="global")),
    # SiLU, ragged shape, a scale per (expert, element), output norm only
    "block_silu_vector": (synth.small_shape(name="block_silu_vector", hidden=80, intermediate=100, top_k=3,
                                            experts=8, tokens=20), 33,
                          dict(activation=0, post_norm=True, down_scale="element")),
    # router input scale (ffn_gate_inp.scale, generation_router.cpp.inc:316-359):
    # the router reads the scaled residual stream; per element with the MoE
    # pre-norm, and one scale for all elements
    "block_router_scale": (synth.small_shape(name="block_router_scale", top_k=3, experts=16, tokens=16), 35,
                           dict(activation=0, pre_norm2=True, router_scale="element")),
    "block_router_scalar": (synth.small_shape(name="block_router_scalar", shared=True, top_k=2, experts=8,
                                              tokens=16), 36,
                            dict(activation=2, unit_offset=True, router_scale="scalar", post_norm=True)),
}


def block_inputs(shape, seed, opts):
    """Seeded block tensors: norm weights ~N(0, 0.3), scales in [0.5, 2),
    the shared gate row bf16 ~N(0, 0.05), hidden ~N(0, 4)."""
    rng = np.random.default_rng(seed)
    H, E = shape.hidden, shape.experts
    vec = lambda: (rng.standard_normal(H) * 0.3).astype(np.float32)
    scale = {"global": 1, "expert": E, "element": E * H}.get(opts.get("down_scale"))
    gate_row = None
    if opts.get("shared_gate_inp"):
        gate_row = ((rng.standard_normal(H) * 0.05).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    blk = oracle.Block(activation=opts.get("activation", 0), unit_offset=opts.get("unit_offset", False),
                       eps=opts.get("eps", 1e-6),
                       pre_norm2=vec() if opts.get("pre_norm2") else None,
                       post_norm1=vec() if opts.get("post_norm1") else None,
                       post_norm2=vec() if opts.get("post_norm2") else None,
                       post_norm=vec() if opts.get("post_norm") else None,
                       down_scale=rng.uniform(0.5, 2.0, scale).astype(np.float32) if scale else None,
                       shared_gate_inp=gate_row)
    rscale = {"scalar": 1, "element": H}.get(opts.get("router_scale"))
    if rscale:
        blk.router_scale = rng.uniform(0.2, 3.0, rscale).astype(np.float32)
    hidden = (rng.standard_normal((shape.tokens, H)) * 2.0).astype(np.float32)
    return blk, hidden


def block_case(name, shape, seed, opts):
    li = synth.make_layer(shape, seed=seed)
    blk, hidden = block_inputs(shape, seed + 1000, opts)
    ref = oracle.Ref(oracle.metadata_json(shape.top_k, norm_topk=shape.norm_topk, block=blk))
    try:
        y, ids, w = ref.moe_block(li, blk, hidden=hidden)
    finally:
        ref.close()
    rec = dict(hidden=shape.hidden, intermediate=shape.intermediate, experts=shape.experts, top_k=shape.top_k,
               tokens=shape.tokens, shared=int(shape.shared), norm_topk=int(shape.norm_topk), skew="", seed=seed,
               digest=li.digest(), ids=ids, w=w, y=y, router=li.router, gate=li.gate, up=li.up, down=li.down,
               x=li.x, hidden_in=hidden, activation=blk.activation, unit_offset=int(blk.unit_offset), eps=blk.eps)
    if shape.shared:
        rec.update(shared_gate=li.shared_gate, shared_up=li.shared_up, shared_down=li.shared_down)
    for k in ("pre_norm2", "post_norm1", "post_norm2", "post_norm", "down_scale", "shared_gate_inp", "router_scale"):
        if getattr(blk, k) is not None:
            rec[k] = getattr(blk, k)
    np.savez_compressed(OUT / f"{name}.npz", **rec)
    print(name)


def block_tables():
    """Known answers of the reference's gated activations (GELU erf and tanh
    forms) and of its RMSNorm, plain and with the Gemma unit offset."""
    rng = np.random.default_rng(34)
    xs = np.concatenate([rng.standard_normal(300).astype(np.float32) * 5,
                         np.array([0.0, -0.0, 20.0, -20.0, 1e-30, -1e-30, 9.0, -9.0], np.float32)])
    ups = rng.standard_normal(xs.size).astype(np.float32)
    norm_in = [(rng.standard_normal(n) * s).astype(np.float32) for n, s in ((64, 1.0), (80, 30.0), (7, 1e-3))]
    norm_w = [(rng.standard_normal(v.size) * 0.3).astype(np.float32) for v in norm_in]
    rec = dict(act_x=xs, act_up=ups)
    ref = oracle.Ref(oracle.metadata_json(2))
    gemma = oracle.Ref(oracle.metadata_json(2, block=oracle.Block(unit_offset=True)))
    try:
        for mode in (0, 1, 2):
            rec[f"act{mode}"] = np.array([ref.lib.ref_gated_activation(mode, float(a), float(u))
                                          for a, u in zip(xs, ups)], np.float32)
        P = lambda a: a.ctypes.data_as(oracle._f32p)
        for i, (v, w) in enumerate(zip(norm_in, norm_w)):
            for tag, r in (("plain", ref), ("unit", gemma)):
                out = np.zeros_like(v)
                assert r.lib.ref_rmsnorm(r.engine, P(w), v.size, P(v), 1e-6, P(out))
                rec[f"norm{i}_{tag}"] = out
            rec[f"norm{i}_in"], rec[f"norm{i}_w"] = v, w
    finally:
        ref.close()
        gemma.close()
    np.savez_compressed(OUT / "block_tables.npz", **rec)
    print("block_tables")


def grouping_case():
    rng = np.random.default_rng(11)
    n = 300
    token = rng.integers(0, 60, n).astype(np.uint32)
    expert = rng.integers(0, 12, n).astype(np.uint32)
    layer = rng.integers(0, 2, n).astype(np.uint32)
    score = rng.random(n).astype(np.float32)
    ref = oracle.Ref("{}")
    try:
        ok, out, batches, cnt = ref.group_tokens(token, expert, score, layer)
    finally:
        ref.close()
    sorted_ = np.array([(a.token_index, a.layer, a.expert) for a in out], np.uint32)
    sorted_score = np.array([a.router_score for a in out], np.float32)
    b = np.array([(x.layer, x.expert, x.first_sorted_index, x.token_count) for x in batches[:cnt]], np.uint32)
    np.savez_compressed(OUT / "grouping.npz", token=token, expert=expert, layer=layer, score=score,
                        ok=ok, sorted=sorted_, sorted_score=sorted_score, batches=b)
    print("grouping", cnt, "batches")


def decode_tables():
    ref = oracle.Ref("{}")
    try:
        e8m0 = np.array([ref.lib.ref_e8m0_to_f32(v) for v in range(256)], np.float32)
        e2m1 = np.array([ref.lib.ref_mxfp4_value(c) for c in range(16)], np.float32)
        rng = np.random.default_rng(12)
        silu_x = np.concatenate([rng.standard_normal(200).astype(np.float32) * 6,
                                 np.array([0.0, -0.0, 88.0, -88.0, 1e-30, -100.0], np.float32)])
        silu_y = np.array([ref.lib.ref_silu(float(v)) for v in silu_x], np.float32)
    finally:
        ref.close()
    np.savez_compressed(OUT / "decode_tables.npz", e8m0=e8m0, e2m1=e2m1, silu_x=silu_x, silu_y=silu_y)
    print("decode_tables")


def provenance():
    """Records what the fixtures' bits depend on: the compiler and -march of
    the reference build (oracle/Makefile) and the host's FMA/AVX2 support
    (the reference's dot products take their AVX2 + FMA branches)."""
    import json
    import platform
    import re
    import subprocess
    mk = (ROOT / "oracle" / "Makefile").read_text()
    march = re.search(r"^MARCH \?= (.*)$", mk, re.M).group(1).strip()
    cxx = subprocess.run(["g++", "--version"], capture_output=True, text=True).stdout.splitlines()[0]
    flags, model = set(), ""
    for line in Path("/proc/cpuinfo").read_text().splitlines():
        if line.startswith("flags") and not flags:
            flags = set(line.split(":", 1)[1].split())
        if line.startswith("model name") and not model:
            model = line.split(":", 1)[1].strip()
    rec = {"compiler": cxx, "march": march, "cxxflags": "-std=c++17 -O3 -DNDEBUG -pthread",
           "host_cpu": model, "machine": platform.machine(),
           "host_flags": {f: f in flags for f in ("avx2", "fma", "f16c", "avx512f")}}
    (OUT / "provenance.json").write_text(json.dumps(rec, indent=1) + "\n")
    print("provenance", rec["march"], rec["host_flags"])


def main(only=None):
    """Writes every fixture, or only those whose name starts with `only`,
    and the record of the build they came from."""
    if not oracle.REF_SO.exists():
        oracle.build(ref=True)
    provenance()
    want = (lambda n: only is None or n.startswith(only))
    if want("decode_tables"):
        decode_tables()
    if want("grouping"):
        grouping_case()
    if want("router_sigmoid"):
        sigmoid_case()
    for name, args in GROUP_LIMIT_CASES.items():
        if want(name):
            group_limit_case(name, *args)
    for name, (shape, seed, tokens, store) in LAYER_CASES.items():
        if want("layer_" + name):
            layer_case(name, shape, seed, tokens, store)
    for name, (shape, seed, opts) in BLOCK_CASES.items():
        if want(name):
            block_case(name, shape, seed, opts)
    if want("block_tables"):
        block_tables()


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
