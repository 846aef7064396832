"""The allocation-free grouping entry point, through the C ABI.

moe_b200_group_tokens_by_expert_noalloc serves callers that cannot allocate
device memory while they run: an engine whose residency cache owns the VRAM
budget has no spare bytes for a mid-layer cudaMalloc.  Its scratch is a fixed
device array inside the library, so this test checks that two calls in a row
-- the second reusing the array the first one filled -- match the allocating
entry point exactly, that a warmed-up call leaves the device's free memory
unchanged, that more batches than max_batches returns 0 with the full count
and the leading batches (as the reference does), and that oversized input is
refused with a message.  The file is collected last so a failure here never
hides another test's result; it also passes on its own in a fresh process.
"""
import ctypes as C
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _lib():
    pkg = ROOT / "storage.llm_b200"
    if "moe_b200" not in sys.modules:
        spec = importlib.util.spec_from_file_location("moe_b200", pkg / "__init__.py",
                                                      submodule_search_locations=[str(pkg)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["moe_b200"] = mod
        spec.loader.exec_module(mod)
    import moe_b200.lib as L
    return L


def _assignments(L, rng, n, token_hi, expert_hi, layer_hi):
    a = (L.Assignment * n)()
    tok = rng.integers(0, token_hi, n)
    ex = rng.integers(0, expert_hi, n)
    ly = rng.integers(0, layer_hi, n)
    sc = rng.random(n).astype(np.float32)
    for i in range(n):
        a[i] = L.Assignment(int(tok[i]), int(ly[i]), int(ex[i]), float(sc[i]))
    return a


def _run(L, fn, a, n, with_err, max_batches=None):
    max_batches = n if max_batches is None else max_batches
    out = (L.Assignment * n)()
    batches = (L.Batch * max(max_batches, 1))()
    cnt = C.c_uint32(0)
    args = [a, n, out, batches, max_batches, C.byref(cnt)]
    if with_err:
        err = C.create_string_buffer(L.ERR_LEN)
        args.append(err)
    ok = fn(*args)
    sorted_ = np.array([(x.token_index, x.layer, x.expert, x.router_score) for x in out], np.float64)
    b = np.array([(x.layer, x.expert, x.first_sorted_index, x.token_count)
                  for x in batches[:min(cnt.value, max_batches)]], np.uint32)
    return ok, sorted_, b, cnt.value


def test_noalloc_grouping_matches_allocating_entry_point_twice():
    L = _lib()
    lib = L.load()
    rng = np.random.default_rng(2024)
    # two different calls in a row: the second reuses the scratch the first
    # filled (larger keys exercise every radix digit)
    cases = [(7000, 50000, 300, 4), (1300, 1 << 31, 70000, 2)]
    for n, tok_hi, ex_hi, ly_hi in cases:
        a = _assignments(L, rng, n, tok_hi, ex_hi, ly_hi)
        ok1, s1, b1, c1 = _run(L, lib.moe_b200_group_tokens_by_expert_noalloc, a, n, True)
        ok2, s2, b2, c2 = _run(L, lib.moe_b200_group_tokens_by_expert, a, n, False)
        assert ok1 == 1 and ok2 == 1
        assert c1 == c2
        assert np.array_equal(s1, s2)
        assert np.array_equal(b1, b2)
        # sorted by (layer, expert, token), batches are the runs
        keys = s1[:, [1, 2, 0]]
        assert all(tuple(keys[i]) <= tuple(keys[i + 1]) for i in range(n - 1))
        assert int(b1[:, 3].sum()) == n


def test_noalloc_rejects_oversized_input():
    L = _lib()
    lib = L.load()
    n = 65536 + 1
    a = (L.Assignment * n)()
    cnt = C.c_uint32(5)
    err = C.create_string_buffer(L.ERR_LEN)
    ok = lib.moe_b200_group_tokens_by_expert_noalloc(a, n, None, None, 0, C.byref(cnt), err)
    assert ok == 0 and cnt.value == 0
    assert b"exceed" in err.value


def test_noalloc_call_allocates_no_device_memory():
    import torch
    L = _lib()
    lib = L.load()
    rng = np.random.default_rng(7)
    n = 20000
    a = _assignments(L, rng, n, 1 << 20, 2000, 3)
    ok, _, _, _ = _run(L, lib.moe_b200_group_tokens_by_expert_noalloc, a, n, True)  # warm-up (module load)
    assert ok == 1
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(torch.cuda.current_device())
    for _ in range(3):
        ok, _, _, _ = _run(L, lib.moe_b200_group_tokens_by_expert_noalloc, a, n, True)
        assert ok == 1
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(torch.cuda.current_device())
    assert free1 == free0, (free0, free1)


def test_noalloc_more_batches_than_room():
    L = _lib()
    lib = L.load()
    rng = np.random.default_rng(11)
    n = 3000
    a = _assignments(L, rng, n, 500, 64, 1)
    _, s_ref, b_ref, c_ref = _run(L, lib.moe_b200_group_tokens_by_expert, a, n, False)
    room = c_ref // 2
    ok, s1, b1, c1 = _run(L, lib.moe_b200_group_tokens_by_expert_noalloc, a, n, True, max_batches=room)
    assert ok == 0 and c1 == c_ref  # the reference's contract: 0, with the full batch count
    assert np.array_equal(s1, s_ref)
    assert np.array_equal(b1, b_ref[:room])
