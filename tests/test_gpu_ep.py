"""Expert-parallel forward on two GPUs (moe_b200_ep_layer_forward: rows
exchanged by this library's kernels over NVLink peer memory).

Each rank owns half of the experts and feeds its own tokens; its output must
match the CPU oracle's layer on those tokens under the same bars as the
single-device tests (routing bit-exact, output within tolerance).  Cases
cover a decode-sized batch, an idle rank (no tokens, still serving its
experts) with the shared expert, a batch past the single-block permutation
limit, a replicated placement, and the dimensions of the largest benchmark
configuration (H=7168, 256 experts, top-8, shared expert; 128 experts per
rank).  Skipped with fewer than two GPUs.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
MAX_ABS = 2e-2
MEAN_REL = 1e-2


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank_main(rank, uid, case, q):
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    from conftest import load_pkg
    import oracle as O

    load_pkg()
    import moe_b200.lib as L
    import moe_b200.synth as synth

    H, I, E, K, tokens, shared = case[:6]
    placement = case[6] if len(case) > 6 else None
    shape = synth.small_shape(name="ep", hidden=H, intermediate=I, experts=E, top_k=K, tokens=8, shared=shared)
    li = synth.make_layer(shape, seed=23)
    T = tokens[rank]
    x = synth.gen_tokens(shape, T, seed=500 + rank, mu=None) if T else np.zeros((0, H), np.uint16)
    eng = L.Engine(rank)
    try:
        eng.ep_init(rank, WORLD, uid)
        if placement:
            eng.ep_set_placement(placement)
        eng.upload_layer_ep(li)
        cfg = L.Engine.cfg(shape, gemm_path=L.GEMM_BLOCKSCALED)
        out = eng.ep_forward_host(cfg, x)
        sent, recv = eng.ep_last_counts(WORLD)
        res = dict(rank=rank, sent=sent.tolist(), recv=recv.tolist())
        if T:
            y_ref, ids_ref, w_ref, _ = O.Port().moe_layer(li, x)
            d = np.abs(out["y_f32"].astype(np.float64) - y_ref)
            res.update(ids_ok=bool(np.array_equal(out["ids"], ids_ref)),
                       w_ok=bool(np.array_equal(out["w"].view(np.uint32), w_ref.view(np.uint32))),
                       max_abs=float(d.max()), mean_rel=float(d.mean() / max(np.abs(y_ref).mean(), 1e-30)))
        q.put(res)
    except Exception as e:  # report, then let the parent fail the test
        q.put(dict(rank=rank, error=repr(e)))
        raise
    finally:
        eng.close()


# expert 0 replicated on both ranks, the rest spread out of order
REPLICATED = [[0, 1], [1], [0], [1], [1], [0], [0], [1]]
CASES = [
    (256, 320, 8, 2, (40, 40), False),
    (256, 320, 8, 3, (64, 0), True),
    (128, 128, 8, 4, (2100, 700), False),
    (256, 320, 8, 3, (96, 80), True, REPLICATED),
    (7168, 2048, 256, 8, (48, 40), True),
]


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("case", CASES, ids=["decode", "idle_rank_shared", "past_single_block_sort",
                                            "replicated_placement", "config4_dims"])
def test_expert_parallel_forward_matches_oracle(case):
    import multiprocessing as mp
    from conftest import load_pkg

    load_pkg()
    import moe_b200.lib as L

    uid = L.Engine.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, uid, case, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=240) for _ in range(WORLD)), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=120)
    for r in results:
        assert "error" not in r, r
    for p in procs:
        assert p.exitcode == 0
    tokens, K = case[4], case[3]
    # every assignment crossed once each way
    assert sum(sum(r["sent"]) for r in results) == sum(tokens) * K
    assert results[0]["sent"][1] == results[1]["recv"][0] and results[1]["sent"][0] == results[0]["recv"][1]
    for r in results:
        if tokens[r["rank"]]:
            assert r["ids_ok"] and r["w_ok"], r
            assert r["max_abs"] <= MAX_ABS and r["mean_rel"] <= MEAN_REL, r


def _absent_rank_main(rank, uid, q, done):
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from conftest import load_pkg

    load_pkg()
    import moe_b200.lib as L
    import moe_b200.synth as synth

    shape = synth.small_shape(hidden=256, intermediate=320, experts=8, top_k=2, tokens=40)
    li = synth.make_layer(shape, seed=29)
    x = synth.gen_tokens(shape, 40, seed=700 + rank, mu=None)
    eng = L.Engine(rank)
    try:
        eng.ep_init(rank, WORLD, uid)
        eng.upload_layer_ep(li)
        cfg = L.Engine.cfg(shape, gemm_path=L.GEMM_BLOCKSCALED)
        eng.ep_forward_host(cfg, x)  # both ranks: buffers sized, peers mapped
        if rank == 0:
            # rank 1 stays away from this call: every device barrier gives up
            # after its bounded wait and the call reports it
            try:
                eng.ep_forward_host(cfg, x)
                msg = "no error"
            except L.MoEError as e:
                msg = str(e)
            eng.sync()  # the error was reported once; the context still works
            q.put(dict(rank=0, msg=msg))
            done.set()
        else:
            done.wait(timeout=120)  # keep the buffers mapped until rank 0 is done
            q.put(dict(rank=1))
    except Exception as e:
        q.put(dict(rank=rank, error=repr(e)))
        done.set()
        raise
    finally:
        eng.close()


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
def test_absent_rank_times_out_with_an_error():
    """A rank that skips a collective call: the other rank's count exchange and
    barriers wait about a second each, record the timeout and return; the call
    fails with that message instead of hanging, and the context stays usable."""
    import multiprocessing as mp
    from conftest import load_pkg

    load_pkg()
    import moe_b200.lib as L

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = L.Engine.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    procs = [ctx.Process(target=_absent_rank_main, args=(r, uid, q, done)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=240) for _ in range(WORLD)), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=120)
    for r in results:
        assert "error" not in r, r
    for p in procs:
        assert p.exitcode == 0
    assert "another rank timed out" in results[0]["msg"], results[0]
