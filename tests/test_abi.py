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
              ("moe_b200_batch_t", L.Batch), ("moe_b200_init_t", L.InitT)]
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
