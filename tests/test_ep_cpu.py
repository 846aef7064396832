"""Expert-parallel layer design on CPU ranks (gloo, world size 2).

The exchange moe_b200_ep_layer_forward runs over NVLink peer stores (this
library's own kernels), restated here over gloo collectives with the oracle
as the per-rank compute: each rank routes its own tokens, sorts the
assignments stably by owner rank (experts in contiguous blocks of E/world),
sends every assignment's token row and its owner-local expert index with an
all-to-allv, the owners run the expert triplet on the rows they receive, the
rows return to their sources at the positions they were sent from, and each
source combines shared + sum_j w_j * y_j in router order.  The result must
equal the single-process oracle layer for each rank's tokens.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fma32(a, b, c):
    # a*b is exact in float64 (24 + 24 significant bits); one more rounding
    # to float64 before the float32 rounding is exact for these magnitudes
    return (np.float64(a) * np.float64(b) + np.float64(c)).astype(np.float32)


def _triplet(port, li, e, xrow):
    H, I = li.shape.hidden, li.shape.intermediate
    if e < 0:
        g, u, d = li.shared_gate, li.shared_up, li.shared_down
    else:
        g, u, d = li.gate[e], li.up[e], li.down[e]
    f32p = C.POINTER(C.c_float)
    u8p = C.POINTER(C.c_uint8)
    g, u, d = (np.ascontiguousarray(a, dtype=np.uint8) for a in (g, u, d))
    xr = np.ascontiguousarray(xrow, dtype=np.float32)
    sg, su, out = np.zeros(I, np.float32), np.zeros(I, np.float32), np.zeros(H, np.float32)
    ok = port.lib.mo_expert_triplet(g.ctypes.data_as(u8p), u.ctypes.data_as(u8p), d.ctypes.data_as(u8p),
                                    xr.ctypes.data_as(f32p), H, I, sg.ctypes.data_as(f32p),
                                    su.ctypes.data_as(f32p), out.ctypes.data_as(f32p))
    assert ok
    return out


def _rank_main(rank, port_no, tokens_per_rank, shared, result_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import torch
    import torch.distributed as dist
    from conftest import load_pkg
    import oracle as O

    load_pkg()
    import moe_b200.synth as synth

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port_no}", rank=rank, world_size=WORLD)
    try:
        shape = synth.small_shape(hidden=64, intermediate=96, experts=8, top_k=3, tokens=8, shared=shared)
        li = synth.make_layer(shape, seed=17)
        T = tokens_per_rank[rank]
        x = synth.gen_tokens(shape, T, seed=300 + rank, mu=None) if T else np.zeros((0, shape.hidden), np.uint16)
        port = O.Port()
        E, K, H = shape.experts, shape.top_k, shape.hidden
        e_per = E // WORLD
        if T:
            ids, w, _, _ = port.router_topk(li, x)
        else:
            ids, w = np.zeros((0, K), np.int32), np.zeros((0, K), np.float32)
        # dispatch: stable order by owner rank
        a = np.arange(T * K)
        owner = ids.ravel() // e_per
        order = a[np.lexsort((a, owner))]
        send_cnt = np.bincount(owner, minlength=WORLD).astype(np.int64)
        pos = np.empty(T * K, np.int64)
        pos[order] = np.arange(T * K)
        xf = O.bf16_to_f32(x) if T else np.zeros((0, H), np.float32)
        send_rows = xf[order // K] if T else np.zeros((0, H), np.float32)
        send_meta = (ids.ravel()[order] % e_per).astype(np.int64) if T else np.zeros(0, np.int64)
        recv_cnt = torch.zeros(WORLD, dtype=torch.int64)
        dist.all_to_all_single(recv_cnt, torch.from_numpy(send_cnt))
        recv_cnt = recv_cnt.numpy()
        n_recv = int(recv_cnt.sum())
        recv_rows = torch.zeros((n_recv, H), dtype=torch.float32)
        dist.all_to_all_single(recv_rows, torch.from_numpy(np.ascontiguousarray(send_rows, np.float32)),
                               recv_cnt.tolist(), send_cnt.tolist())
        recv_meta = torch.zeros(n_recv, dtype=torch.int64)
        dist.all_to_all_single(recv_meta, torch.from_numpy(send_meta), recv_cnt.tolist(), send_cnt.tolist())
        # owners: local experts on the received rows
        e0 = rank * e_per
        y_loc = np.stack([_triplet(port, li, e0 + int(m), r) for m, r in
                          zip(recv_meta.numpy(), recv_rows.numpy())]) if n_recv else np.zeros((0, H), np.float32)
        ret = torch.zeros((T * K, H), dtype=torch.float32)
        dist.all_to_all_single(ret, torch.from_numpy(np.ascontiguousarray(y_loc, np.float32)), send_cnt.tolist(),
                               recv_cnt.tolist())
        ret = ret.numpy()
        # combine at the source: shared first, then router order
        y = np.zeros((T, H), np.float32)
        for t in range(T):
            acc = np.zeros(H, np.float32)
            if shared:
                acc = (acc + _triplet(port, li, -1, xf[t]) * np.float32(1.0)).astype(np.float32)
            for j in range(K):
                acc = _fma32(w[t, j], ret[pos[t * K + j]], acc)
            y[t] = acc
        if T:
            y_ref, ids_ref, w_ref, _ = port.moe_layer(li, x, threads=1)
            result_q.put((rank, bool(np.array_equal(ids, ids_ref)), float(np.abs(y - y_ref).max()),
                          float(np.abs(y_ref).max()), n_recv))
        else:
            result_q.put((rank, True, 0.0, 0.0, n_recv))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,shared", [((6, 5), False), ((7, 0), True)], ids=["uneven", "idle_rank_shared"])
def test_expert_parallel_exchange_matches_single_process(tokens, shared):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_no = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port_no, tokens, shared, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total_recv = 0
    for rank, ids_ok, err, scale, n_recv in results:
        assert ids_ok, rank
        assert err <= 1e-6 * max(scale, 1e-3), (rank, err, scale)
        total_recv += n_recv
    assert total_recv == sum(tokens) * 3
