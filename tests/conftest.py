import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
PKG_DIR = ROOT / "storage.llm_b200"
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def load_pkg():
    """The package directory is named storage.llm_b200 (not an identifier),
    so it is registered under the import name `moe_b200`."""
    if "moe_b200" in sys.modules:
        return sys.modules["moe_b200"]
    spec = importlib.util.spec_from_file_location("moe_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def synth(pkg):
    import moe_b200.synth as s
    return s


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    if not oracle.PORT_SO.exists():
        oracle.build(ref=False)
    return oracle


@pytest.fixture(scope="session")
def port(oracle_mod):
    return oracle_mod.Port()


def golden(name):
    return dict(np.load(GOLDEN / name, allow_pickle=False))


def layer_from_golden(synth, g):
    """Rebuilds a LayerInputs from a golden record (stored inputs, or the
    seed whose regenerated inputs must match the recorded digest)."""
    shape = synth.LayerShape("golden", int(g["hidden"]), int(g["intermediate"]), int(g["experts"]),
                             int(g["top_k"]), int(g["tokens"]), bool(int(g["shared"])),
                             str(g["skew"]) or None, bool(int(g["norm_topk"])))
    if "x" in g:
        li = synth.LayerInputs(shape, g["router"], g["gate"], g["up"], g["down"], g["x"])
        if shape.shared:
            li.shared_gate, li.shared_up, li.shared_down = g["shared_gate"], g["shared_up"], g["shared_down"]
    else:
        li = synth.make_layer(shape, seed=int(g["seed"]), tokens=int(g["tokens"]))
    assert li.digest() == str(g["digest"]), "regenerated inputs differ from the golden record"
    return li


BLOCK_PARTS = ("pre_norm2", "post_norm1", "post_norm2", "post_norm", "down_scale", "shared_gate_inp", "router_scale")


def block_from_golden(oracle_mod, g):
    """The block options and residual-stream input of a block fixture."""
    blk = oracle_mod.Block(activation=int(g["activation"]), unit_offset=bool(int(g["unit_offset"])),
                           eps=float(g["eps"]), **{k: g[k] for k in BLOCK_PARTS if k in g})
    return blk, g["hidden_in"]
