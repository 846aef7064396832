"""The benchmark configurations at full size through the CUDA path.

The whole oracle layer at these sizes is hours of CPU work, so the checks are
the ones whose cost does not grow with the batch, plus a seeded sample:
  * permutation: exactly the reference grouping order
    (moe_pc_group_tokens_by_expert, token_grouping.cpp.inc:47-55) over every
    assignment of the batch, and per-expert counts equal to the routed ids;
  * router scores, ids and weights of a seeded token sample: bit-exact
    against the oracle (tokens are routed independently);
  * layer output of the same sample: max abs err <= 2e-2 and mean rel err
    <= 1e-2 against the oracle layer run on those tokens alone (a token's
    output does not depend on the other tokens of the batch).
Inputs are the bench's own (synth.make_layer(shape, seed=0, tokens=T)).
Config 4 (16,384 tokens of H = 7168, 256 experts, top-8, one shared expert)
is the largest; the test prints the sample's measured error for the fp32 and
bf16 outputs.  The bf16 output is checked as the rounding of the fp32 output
(bf16's own half-ulp at |y| >= 8 exceeds the absolute bar).
"""
import numpy as np
import pytest

from test_gpu_layer import check_bf16_output

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-2
SAMPLE = 24


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def errors(y, ref):
    d = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    return float(d.max()), float(d.mean() / max(np.abs(ref).mean(), 1e-30))


@pytest.fixture(scope="module")
def L(pkg):
    import moe_b200.lib as lib
    return lib


@pytest.fixture(scope="module")
def engine(L):
    e = L.Engine(0)
    yield e
    e.close()


def full_size_tokens(synth, config):
    shape = synth.CONFIGS[config]
    return 256 if config == 1 else (shape.tokens or sum(synth.prefill_lengths()))


def token_sample(config, tokens):
    rng = np.random.default_rng(100 + config)
    return np.sort(rng.choice(tokens, size=min(SAMPLE, tokens), replace=False))


@pytest.mark.parametrize("config", [1, 3, 2, 4], ids=["c1_decode_t256", "c3_t4096", "c2_prefill_8k", "c4_t16384"])
def test_full_size_configuration(engine, synth, L, port, config):
    shape = synth.CONFIGS[config]
    T = full_size_tokens(synth, config)
    K, E = shape.top_k, shape.experts
    li = synth.make_layer(shape, seed=0, tokens=T)
    engine.upload_layer(li)
    out = engine.forward_host(L.Engine.cfg(shape), li.x)
    ids = out["ids"]

    a = np.arange(T * K)
    want = a[np.lexsort((a // K, ids.ravel()))]
    assert np.array_equal(out["perm"], want.astype(np.uint32))
    counts = engine.read(L.BUF_GROUP_COUNT, (E,), np.uint32)
    assert np.array_equal(counts, np.bincount(ids.ravel(), minlength=E))

    sample = token_sample(config, T)
    xs = li.x[sample]
    ids_ref, w_ref, scores_ref, ties = port.router_topk(li, x=xs)
    assert ties == 0
    scores = engine.read(L.BUF_SCORES, (T, E), np.float32)
    assert np.array_equal(bits(scores[sample]), bits(scores_ref))
    assert np.array_equal(ids[sample], ids_ref)
    assert np.array_equal(bits(out["w"][sample]), bits(w_ref))
    y_ref, _, _, _ = port.moe_layer(li, x=xs)
    mx, mr = errors(out["y_f32"][sample], y_ref)
    y16 = (out["y_bf16"][sample].astype(np.uint32) << 16).view(np.float32)
    mx16, mr16 = errors(y16, y_ref)
    print(f"config {config}: sample of {len(sample)} tokens, fp32 output max abs {mx:.3e} mean rel {mr:.3e}; "
          f"bf16 output max abs {mx16:.3e} mean rel {mr16:.3e}")
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    check_bf16_output(out["y_bf16"][sample], out["y_f32"][sample], y_ref)
