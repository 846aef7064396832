"""The C-ABI library builds for sm_100a, loads without a GPU and exports
every entry point include/moe_b200.h declares (no compute calls here)."""
import ctypes
from pathlib import Path

import pytest


@pytest.fixture(scope="module")
def lib(pkg):
    import moe_b200.build as build
    import moe_b200.lib as L
    build.build()
    return L.load()


def test_header_declares_the_boundary(pkg):
    import moe_b200.lib as L
    names = set(L.header_symbols())
    for required in ("moe_b200_create", "moe_b200_destroy", "moe_b200_upload_router", "moe_b200_upload_expert",
                     "moe_b200_layer_forward", "moe_b200_layer_forward_host", "moe_b200_sync",
                     "moe_b200_run_expert_triplet_f32", "moe_b200_group_tokens_by_expert"):
        assert required in names


def test_library_exports_every_declared_symbol(lib, pkg):
    import moe_b200.lib as L
    for name in L.header_symbols():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_struct_layouts(pkg, tmp_path):
    """The ctypes mirrors have the header's sizes and field offsets (checked
    by compiling include/moe_b200.h with the host C compiler)."""
    import shutil
    import subprocess
    import moe_b200.lib as L
    assert ctypes.sizeof(L.Assignment) == 16 and ctypes.sizeof(L.Batch) == 16
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    inc = Path(__file__).resolve().parents[1] / "include"
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "moe_b200.h"', "int main(void) {"]
    checks = [("moe_b200_layer_cfg_t", L.LayerCfg), ("moe_b200_assignment_t", L.Assignment),
              ("moe_b200_batch_t", L.Batch), ("moe_b200_init_t", L.InitT),
              ("moe_b200_block_tensors_t", L.BlockTensors)]
    for cname, py in checks:
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(inc), str(src), "-o", str(exe)], check=True)
    got = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.split("\n") if l)
    for cname, py in checks:
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, (cname, fname)


def test_group_tokens_rejects_empty_input_without_gpu(lib, pkg):
    # argument checks run before any device work (token_grouping.cpp.inc:9-15)
    import moe_b200.lib as L
    cnt = ctypes.c_uint32(7)
    assert lib.moe_b200_group_tokens_by_expert(None, 0, None, None, 0, ctypes.byref(cnt)) == 0
    assert cnt.value == 0


def test_create_without_gpu_fails_loudly(lib, pkg):
    import torch
    import moe_b200.lib as L
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(L.MoEError):
        L.Engine(0)


CPP_CLIENT = r"""
// A C++ caller in the style of the reference engine's binding: create an
// engine, report its error text, no exceptions across the boundary.
#include <cstdio>
#include <cstring>
#include "moe_b200.h"

int main() {
    char err[MOE_B200_ERR_LEN] = {0};
    moe_b200_init_t init{0, 1};
    moe_b200_engine_t* eng = moe_b200_create(&init, err);
    if (!eng) {
        // no B200 here: the library must say why instead of falling back
        std::printf("no-engine:%s\n", err[0] ? err : "(empty)");
        return err[0] ? 0 : 2;
    }
    moe_b200_layer_cfg_t cfg{};
    cfg.hidden = 60;  // not a multiple of 8: rejected before any device work
    cfg.intermediate = 64;
    cfg.experts = 8;
    cfg.top_k = 2;
    const int ok = moe_b200_layer_forward_host(eng, &cfg, nullptr, 1, nullptr, nullptr, nullptr, nullptr,
                                               nullptr, err);
    moe_b200_destroy(eng);
    std::printf("engine:%d:%s\n", ok, err);
    return ok == 0 && err[0] ? 0 : 3;
}
"""


def test_cpp_client_builds_links_and_fails_loudly_without_a_b200(lib, pkg, tmp_path):
    """The header compiles as C++, a client links against the library, and
    without a B200 engine creation fails with a message (no CPU path); on a
    B200 host the same client gets an argument error instead."""
    import shutil
    import subprocess
    import moe_b200.lib as L
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    root = Path(__file__).resolve().parents[1]
    src = tmp_path / "client.cpp"
    src.write_text(CPP_CLIENT)
    exe = tmp_path / "client"
    so = Path(L.LIB_PATH)
    subprocess.run([cxx, "-std=c++17", "-I", str(root / "include"), str(src), "-o", str(exe), str(so),
                    f"-Wl,-rpath,{so.parent}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.startswith(("no-engine:", "engine:0:")), r.stdout
