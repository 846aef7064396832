"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the CPU checkers.

* ``Port``  -> oracle/_ref/libmoe_port.so, this repository's plain-C
  restatement of the reference hot path (oracle/moe_oracle.c);
* ``Ref``   -> oracle/_ref/libmoe_ref.so, the reference's own C++ hot path
  compiled from its sources (oracle/ref_harness.cpp + oracle/Makefile).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline and
reference arms may use this module, and only as the checker or the timed
CPU baseline.  The CUDA product never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
PORT_SO = REF_DIR / "libmoe_port.so"
REF_SO = REF_DIR / "libmoe_ref.so"
# The reference checkout: MOE_REFERENCE_ROOT when set, else a directory named
# "reference" beside this repository's root.  Only builds of the reference
# library need it; without it build() makes the port alone.
REFERENCE_ROOT = Path(os.environ.get("MOE_REFERENCE_ROOT") or (HERE.parent.parent / "reference"))

_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_i32p = C.POINTER(C.c_int32)
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)


def build(ref: bool = True) -> None:
    """Builds the port always, and the reference library when its sources
    are present (they are not on the GPU box, which uses the prebuilt .so)."""
    targets = ["port"]
    if ref and REFERENCE_ROOT.is_dir():
        targets.append("ref")
    subprocess.run(["make", "-s", "-j8", "-C", str(HERE), f"REF={REFERENCE_ROOT}"] + targets,
                   check=True)


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t) if a is not None else None


class MoLayer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("experts", C.c_uint32),
                ("top_k", C.c_uint32), ("score_sigmoid", C.c_int32), ("norm_topk", C.c_int32),
                ("routed_scale", C.c_float), ("router_bf16", _u16p), ("gate", _u8p), ("up", _u8p),
                ("down", _u8p), ("shared_gate", _u8p), ("shared_up", _u8p), ("shared_down", _u8p),
                ("n_group", C.c_uint32), ("topk_group", C.c_uint32),
                ("activation", C.c_int32), ("norm_unit_offset", C.c_int32), ("norm_eps", C.c_float),
                ("pre_norm2", _f32p), ("post_norm1", _f32p), ("post_norm2", _f32p), ("post_norm", _f32p),
                ("down_scale", _f32p), ("down_scale_count", C.c_uint64), ("shared_gate_inp", _u16p),
                ("router_scale", _f32p), ("router_scale_count", C.c_uint64), ("present", _u8p)]


class RefLayer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("experts", C.c_uint32),
                ("top_k", C.c_uint32), ("router_bf16", _u16p), ("gate", _u8p), ("up", _u8p),
                ("down", _u8p), ("shared_gate", _u8p), ("shared_up", _u8p), ("shared_down", _u8p)]


class RefBlock(C.Structure):
    _fields_ = [("base", RefLayer), ("eps", C.c_float), ("pre_norm2", _f32p), ("post_norm1", _f32p),
                ("post_norm2", _f32p), ("post_norm", _f32p), ("down_scale", _f32p),
                ("down_scale_count", C.c_uint64), ("shared_gate_inp", _u16p), ("router_scale", _f32p),
                ("router_scale_count", C.c_uint64)]


class Assignment(C.Structure):
    _fields_ = [("token_index", C.c_uint32), ("layer", C.c_uint32), ("expert", C.c_uint32),
                ("router_score", C.c_float)]


class Batch(C.Structure):
    _fields_ = [("layer", C.c_uint32), ("expert", C.c_uint32), ("first_sorted_index", C.c_uint32),
                ("token_count", C.c_uint32)]


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


@dataclass
class Block:
    """Optional parts of a Gemma-style MoE block around the experts
    (generation_mlp.cpp.inc:94-104, 145-175, 234-250, 380-429, 478-570);
    the defaults are the plain layer.  Norm weights and scales are float32;
    `shared_gate_inp` is a bf16 row (uint16)."""
    activation: int = 0                  # 0 SiLU, 1 GELU (erf), 2 GELU (tanh form)
    unit_offset: bool = False            # RMSNorm by (1 + w): Gemma models
    eps: float = 1e-6
    pre_norm2: Optional[np.ndarray] = None    # [H] routed experts read RMSNorm(hidden)
    post_norm1: Optional[np.ndarray] = None   # [H] shared expert output
    post_norm2: Optional[np.ndarray] = None   # [H] each routed expert's output
    post_norm: Optional[np.ndarray] = None    # [H] block output
    down_scale: Optional[np.ndarray] = None   # [1], [E] or [E*H]
    shared_gate_inp: Optional[np.ndarray] = None  # [H] bf16
    router_scale: Optional[np.ndarray] = None     # [1] or [H]: the router reads scaled hidden

    def metadata(self) -> list[str]:
        """GGUF metadata entries through which the reference learns the
        activation and the unit offset (raw_forward_utils.cpp.inc:322-350)."""
        parts = []
        if self.activation == 2:
            parts.append('"hidden_activation":"gelu_pytorch_tanh"')
        elif self.activation == 1:
            parts.append('"hidden_activation":"gelu"')
        if self.unit_offset:
            parts.append('"general.architecture":"gemma3"')
        return parts


class Port:
    """The C restatement (always available once built)."""

    def __init__(self, path: Path = PORT_SO):
        self.lib = C.CDLL(str(path))
        L = self.lib
        L.mo_e8m0_to_f32.restype = C.c_float
        L.mo_e8m0_to_f32.argtypes = [C.c_uint8]
        L.mo_mxfp4_value.restype = C.c_float
        L.mo_mxfp4_value.argtypes = [C.c_uint8]
        L.mo_mxfp4_dot_row.restype = C.c_float
        L.mo_mxfp4_dot_row.argtypes = [_u8p, _f32p, C.c_uint32]
        L.mo_bf16_dot_row.restype = C.c_float
        L.mo_bf16_dot_row.argtypes = [_u16p, _f32p, C.c_uint32]
        L.mo_silu.restype = C.c_float
        L.mo_silu.argtypes = [C.c_float]
        L.mo_router_scores.argtypes = [C.POINTER(MoLayer), _f32p, _f32p]
        L.mo_router_topk.restype = C.c_int
        L.mo_router_topk.argtypes = [C.POINTER(MoLayer), _f32p, _i32p, _f32p, _u32p]
        L.mo_group_tokens_by_expert.restype = C.c_int
        L.mo_group_tokens_by_expert.argtypes = [C.POINTER(Assignment), C.c_uint32, C.POINTER(Assignment),
                                                C.POINTER(Batch), C.c_uint32, _u32p]
        L.mo_expert_triplet.restype = C.c_int
        L.mo_expert_triplet.argtypes = [_u8p, _u8p, _u8p, _f32p, C.c_uint32, C.c_uint32, _f32p, _f32p, _f32p]
        L.mo_moe_layer.restype = C.c_int
        L.mo_moe_layer.argtypes = [C.POINTER(MoLayer), _u16p, C.c_uint32, _f32p, _i32p, _f32p,
                                   C.c_uint32, _u32p]
        L.mo_moe_block.restype = C.c_int
        L.mo_moe_block.argtypes = [C.POINTER(MoLayer), _u16p, _f32p, C.c_uint32, _f32p, _i32p, _f32p,
                                   C.c_uint32, _u32p]
        L.mo_gated_activation.restype = C.c_float
        L.mo_gated_activation.argtypes = [C.c_int32, C.c_float, C.c_float]
        L.mo_rmsnorm.restype = C.c_int
        L.mo_rmsnorm.argtypes = [_f32p, _f32p, C.c_uint32, C.c_float, C.c_int32, _f32p]

    def _layer(self, li, score_sigmoid=0, norm_topk=None, routed_scale=1.0, n_group=0, topk_group=0,
               present=None):
        """present: E + 1 flags (the last the shared expert), 0 = missing; None = all."""
        s = li.shape
        keep = dict(router=_c(li.router, np.uint16), gate=_c(li.gate, np.uint8), up=_c(li.up, np.uint8),
                    down=_c(li.down, np.uint8), sg=_c(li.shared_gate, np.uint8),
                    su=_c(li.shared_up, np.uint8), sd=_c(li.shared_down, np.uint8),
                    present=_c(present, np.uint8))
        nt = s.norm_topk if norm_topk is None else norm_topk
        L = MoLayer(s.hidden, s.intermediate, s.experts, s.top_k, int(score_sigmoid), int(nt),
                    float(routed_scale), _p(keep["router"], _u16p), _p(keep["gate"], _u8p),
                    _p(keep["up"], _u8p), _p(keep["down"], _u8p), _p(keep["sg"], _u8p),
                    _p(keep["su"], _u8p), _p(keep["sd"], _u8p), int(n_group), int(topk_group))
        L.present = _p(keep["present"], _u8p)
        return L, keep

    def moe_layer(self, li, x=None, threads: int = 0, **kw):
        x = _c(li.x if x is None else x, np.uint16)
        T = x.shape[0]
        L, keep = self._layer(li, **kw)
        H, K = li.shape.hidden, li.shape.top_k
        y = np.zeros((T, H), np.float32)
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        ties = C.c_uint32(0)
        ok = self.lib.mo_moe_layer(C.byref(L), _p(x, _u16p), T, _p(y, _f32p), _p(ids, _i32p), _p(w, _f32p),
                                   threads or (os.cpu_count() or 1), C.byref(ties))
        if not ok:
            raise RuntimeError("oracle layer failed")
        return y, ids, w, ties.value

    def moe_block(self, li, blk: Block, hidden=None, x=None, threads: int = 0, **kw):
        """The layer with the block's optional parts; `hidden` [T x H] f32 is
        the residual stream (needed with pre_norm2).  Returns y (what the
        block adds to hidden), ids, w, ties."""
        x = _c(li.x if x is None else x, np.uint16)
        T = x.shape[0]
        L, keep = self._layer(li, **kw)
        H, K = li.shape.hidden, li.shape.top_k
        keep.update(pn2=_c(blk.pre_norm2, np.float32), n1=_c(blk.post_norm1, np.float32),
                    n2=_c(blk.post_norm2, np.float32), n=_c(blk.post_norm, np.float32),
                    ds=_c(blk.down_scale, np.float32), sgi=_c(blk.shared_gate_inp, np.uint16),
                    rs=_c(blk.router_scale, np.float32), hid=_c(hidden, np.float32))
        L.activation, L.norm_unit_offset, L.norm_eps = int(blk.activation), int(blk.unit_offset), float(blk.eps)
        L.pre_norm2, L.post_norm1 = _p(keep["pn2"], _f32p), _p(keep["n1"], _f32p)
        L.post_norm2, L.post_norm = _p(keep["n2"], _f32p), _p(keep["n"], _f32p)
        L.down_scale = _p(keep["ds"], _f32p)
        L.down_scale_count = 0 if keep["ds"] is None else keep["ds"].size
        L.shared_gate_inp = _p(keep["sgi"], _u16p)
        L.router_scale = _p(keep["rs"], _f32p)
        L.router_scale_count = 0 if keep["rs"] is None else keep["rs"].size
        y = np.zeros((T, H), np.float32)
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        ties = C.c_uint32(0)
        ok = self.lib.mo_moe_block(C.byref(L), _p(x, _u16p), _p(keep["hid"], _f32p), T, _p(y, _f32p),
                                   _p(ids, _i32p), _p(w, _f32p), threads or (os.cpu_count() or 1),
                                   C.byref(ties))
        if not ok:
            raise RuntimeError("oracle block failed")
        return y, ids, w, ties.value

    def router_topk(self, li, x=None, **kw):
        x = _c(li.x if x is None else x, np.uint16)
        L, keep = self._layer(li, **kw)
        T, K, E = x.shape[0], li.shape.top_k, li.shape.experts
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        scores = np.zeros((T, E), np.float32)
        ties = C.c_uint32(0)
        xf = bf16_to_f32(x)
        for t in range(T):
            row = np.ascontiguousarray(xf[t])
            self.lib.mo_router_scores(C.byref(L), _p(row, _f32p), _p(scores[t], _f32p))
            self.lib.mo_router_topk(C.byref(L), _p(row, _f32p), _p(ids[t], _i32p), _p(w[t], _f32p),
                                    C.byref(ties))
        return ids, w, scores, ties.value

    def mxfp4_dot_rows(self, packed: np.ndarray, x: np.ndarray) -> np.ndarray:
        packed = _c(packed, np.uint8)
        x = _c(x, np.float32)
        rows = packed.shape[0]
        out = np.empty(rows, np.float32)
        for r in range(rows):
            out[r] = self.lib.mo_mxfp4_dot_row(_p(packed[r], _u8p), _p(x, _f32p), x.shape[0])
        return out

    def group_tokens(self, token, expert, score=None, layer=None):
        n = len(token)
        a = (Assignment * n)()
        for i in range(n):
            a[i] = Assignment(int(token[i]), 0 if layer is None else int(layer[i]), int(expert[i]),
                              0.0 if score is None else float(score[i]))
        out = (Assignment * n)()
        batches = (Batch * max(n, 1))()
        cnt = C.c_uint32(0)
        ok = self.lib.mo_group_tokens_by_expert(a, n, out, batches, max(n, 1), C.byref(cnt))
        return ok, out, batches, cnt.value


class Ref:
    """The reference's own compiled hot path."""

    def __init__(self, metadata_json: str, path: Path = REF_SO):
        self.lib = C.CDLL(str(path))
        L = self.lib
        L.ref_engine_create.restype = C.c_void_p
        L.ref_engine_create.argtypes = [C.c_char_p]
        L.ref_engine_destroy.argtypes = [C.c_void_p]
        L.ref_row_threads.restype = C.c_uint32
        L.ref_e8m0_to_f32.restype = C.c_float
        L.ref_e8m0_to_f32.argtypes = [C.c_uint8]
        L.ref_mxfp4_value.restype = C.c_float
        L.ref_mxfp4_value.argtypes = [C.c_uint8]
        L.ref_silu.restype = C.c_float
        L.ref_silu.argtypes = [C.c_float]
        L.ref_mxfp4_dot_rows.argtypes = [_u8p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.ref_bf16_dot_rows.argtypes = [_u16p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.ref_router_topk.restype = C.c_int
        L.ref_router_topk.argtypes = [C.c_void_p, _u16p, C.c_uint32, C.c_uint32, _u16p, C.c_uint32,
                                      C.c_uint32, _i32p, _f32p, _f32p]
        L.ref_moe_layer.restype = C.c_int
        L.ref_moe_layer.argtypes = [C.c_void_p, C.POINTER(RefLayer), _u16p, C.c_uint32, _f32p, _i32p, _f32p]
        L.ref_moe_layer_engine.restype = C.c_int
        L.ref_moe_layer_engine.argtypes = [C.c_void_p, C.POINTER(RefLayer), _u16p, C.c_uint32, _f32p, _i32p, _f32p,
                                           C.c_char_p]
        L.ref_moe_layer_engine_present.restype = C.c_int
        L.ref_moe_layer_engine_present.argtypes = [C.c_void_p, C.POINTER(RefLayer), _u16p, C.c_uint32, _f32p, _i32p,
                                                   _f32p, C.c_char_p, _u8p]
        L.ref_moe_block_engine.restype = C.c_int
        L.ref_moe_block_engine.argtypes = [C.c_void_p, C.POINTER(RefBlock), _u16p, _f32p, C.c_uint32, _f32p, _i32p,
                                           _f32p, C.c_char_p]
        L.ref_moe_block.restype = C.c_int
        L.ref_moe_block.argtypes = [C.c_void_p, C.POINTER(RefBlock), _u16p, _f32p, C.c_uint32, _f32p, _i32p,
                                    _f32p]
        L.ref_gated_activation.restype = C.c_float
        L.ref_gated_activation.argtypes = [C.c_int32, C.c_float, C.c_float]
        L.ref_rmsnorm.restype = C.c_int
        L.ref_rmsnorm.argtypes = [C.c_void_p, _f32p, C.c_uint32, _f32p, C.c_float, _f32p]
        L.ref_group_tokens_by_expert.restype = C.c_int
        L.ref_group_tokens_by_expert.argtypes = [C.POINTER(Assignment), C.c_uint32, C.POINTER(Assignment),
                                                 C.POINTER(Batch), C.c_uint32, _u32p]
        self.engine = L.ref_engine_create(metadata_json.encode())
        if not self.engine:
            raise RuntimeError("reference engine create failed")

    def close(self):
        if self.engine:
            self.lib.ref_engine_destroy(self.engine)
            self.engine = None

    def moe_layer(self, li, x=None):
        s = li.shape
        x = _c(li.x if x is None else x, np.uint16)
        T = x.shape[0]
        keep = [_c(li.router, np.uint16), _c(li.gate, np.uint8), _c(li.up, np.uint8), _c(li.down, np.uint8),
                _c(li.shared_gate, np.uint8), _c(li.shared_up, np.uint8), _c(li.shared_down, np.uint8)]
        d = RefLayer(s.hidden, s.intermediate, s.experts, s.top_k, _p(keep[0], _u16p), _p(keep[1], _u8p),
                     _p(keep[2], _u8p), _p(keep[3], _u8p), _p(keep[4], _u8p), _p(keep[5], _u8p),
                     _p(keep[6], _u8p))
        y = np.zeros((T, s.hidden), np.float32)
        ids = np.zeros((T, s.top_k), np.int32)
        w = np.zeros((T, s.top_k), np.float32)
        if not self.lib.ref_moe_layer(self.engine, C.byref(d), _p(x, _u16p), T, _p(y, _f32p), _p(ids, _i32p),
                                      _p(w, _f32p)):
            raise RuntimeError("reference layer failed")
        return y, ids, w

    def moe_layer_engine(self, li, shard_path: str, x=None, present=None):
        """The layer through the reference's moe_layer_moe_mlp_f32 itself, the
        experts as tensor records over a shard file written to shard_path
        (ref_harness.cpp ref_moe_layer_engine); returns y, ids, w.  present:
        E + 1 flags (the last the shared expert), 0 = the expert is missing."""
        s = li.shape
        x = _c(li.x if x is None else x, np.uint16)
        T = x.shape[0]
        keep = [_c(li.router, np.uint16), _c(li.gate, np.uint8), _c(li.up, np.uint8), _c(li.down, np.uint8),
                _c(li.shared_gate, np.uint8), _c(li.shared_up, np.uint8), _c(li.shared_down, np.uint8)]
        d = RefLayer(s.hidden, s.intermediate, s.experts, s.top_k, _p(keep[0], _u16p), _p(keep[1], _u8p),
                     _p(keep[2], _u8p), _p(keep[3], _u8p), _p(keep[4], _u8p), _p(keep[5], _u8p),
                     _p(keep[6], _u8p))
        y = np.zeros((T, s.hidden), np.float32)
        ids = np.zeros((T, s.top_k), np.int32)
        w = np.zeros((T, s.top_k), np.float32)
        if present is None:
            ok = self.lib.ref_moe_layer_engine(self.engine, C.byref(d), _p(x, _u16p), T, _p(y, _f32p),
                                               _p(ids, _i32p), _p(w, _f32p), str(shard_path).encode())
        else:
            pr = _c(present, np.uint8)
            ok = self.lib.ref_moe_layer_engine_present(self.engine, C.byref(d), _p(x, _u16p), T, _p(y, _f32p),
                                                       _p(ids, _i32p), _p(w, _f32p), str(shard_path).encode(),
                                                       _p(pr, _u8p))
        if not ok:
            raise RuntimeError("reference layer function failed")
        return y, ids, w

    def moe_block(self, li, blk: Block, hidden=None, x=None, shard_path=None):
        """The block with its optional parts (the engine's metadata must
        carry blk.metadata()); returns y (what the block adds to hidden),
        ids, w.  With shard_path, through the reference's
        moe_layer_moe_mlp_f32 itself (ref_moe_block_engine), else the leaf
        composition (ref_moe_block)."""
        s = li.shape
        x = _c(li.x if x is None else x, np.uint16)
        T = x.shape[0]
        keep = [_c(li.router, np.uint16), _c(li.gate, np.uint8), _c(li.up, np.uint8), _c(li.down, np.uint8),
                _c(li.shared_gate, np.uint8), _c(li.shared_up, np.uint8), _c(li.shared_down, np.uint8),
                _c(blk.pre_norm2, np.float32), _c(blk.post_norm1, np.float32), _c(blk.post_norm2, np.float32),
                _c(blk.post_norm, np.float32), _c(blk.down_scale, np.float32),
                _c(blk.shared_gate_inp, np.uint16), _c(hidden, np.float32), _c(blk.router_scale, np.float32)]
        base = RefLayer(s.hidden, s.intermediate, s.experts, s.top_k, _p(keep[0], _u16p), _p(keep[1], _u8p),
                        _p(keep[2], _u8p), _p(keep[3], _u8p), _p(keep[4], _u8p), _p(keep[5], _u8p),
                        _p(keep[6], _u8p))
        d = RefBlock(base, float(blk.eps), _p(keep[7], _f32p), _p(keep[8], _f32p), _p(keep[9], _f32p),
                     _p(keep[10], _f32p), _p(keep[11], _f32p), 0 if keep[11] is None else keep[11].size,
                     _p(keep[12], _u16p), _p(keep[14], _f32p), 0 if keep[14] is None else keep[14].size)
        y = np.zeros((T, s.hidden), np.float32)
        ids = np.zeros((T, s.top_k), np.int32)
        w = np.zeros((T, s.top_k), np.float32)
        if shard_path is not None:
            ok = self.lib.ref_moe_block_engine(self.engine, C.byref(d), _p(x, _u16p), _p(keep[13], _f32p), T,
                                               _p(y, _f32p), _p(ids, _i32p), _p(w, _f32p), str(shard_path).encode())
        else:
            ok = self.lib.ref_moe_block(self.engine, C.byref(d), _p(x, _u16p), _p(keep[13], _f32p), T,
                                        _p(y, _f32p), _p(ids, _i32p), _p(w, _f32p))
        if not ok:
            raise RuntimeError("reference block failed")
        return y, ids, w

    def router_topk(self, li, x=None):
        s = li.shape
        x = _c(li.x if x is None else x, np.uint16)
        router = _c(li.router, np.uint16)
        T = x.shape[0]
        ids = np.zeros((T, s.top_k), np.int32)
        w = np.zeros((T, s.top_k), np.float32)
        scores = np.zeros((T, s.experts), np.float32)
        if not self.lib.ref_router_topk(self.engine, _p(router, _u16p), s.experts, s.hidden, _p(x, _u16p), T,
                                        s.top_k, _p(ids, _i32p), _p(w, _f32p), _p(scores, _f32p)):
            raise RuntimeError("reference router failed")
        return ids, w, scores

    def mxfp4_dot_rows(self, packed, x):
        packed = _c(packed, np.uint8)
        x = _c(x, np.float32)
        out = np.empty(packed.shape[0], np.float32)
        self.lib.ref_mxfp4_dot_rows(_p(packed, _u8p), packed.shape[0], x.shape[0], _p(x, _f32p), _p(out, _f32p))
        return out

    def bf16_dot_rows(self, w, x):
        w = _c(w, np.uint16)
        x = _c(x, np.float32)
        out = np.empty(w.shape[0], np.float32)
        self.lib.ref_bf16_dot_rows(_p(w, _u16p), w.shape[0], w.shape[1], _p(x, _f32p), _p(out, _f32p))
        return out

    def group_tokens(self, token, expert, score=None, layer=None):
        n = len(token)
        a = (Assignment * n)()
        for i in range(n):
            a[i] = Assignment(int(token[i]), 0 if layer is None else int(layer[i]), int(expert[i]),
                              0.0 if score is None else float(score[i]))
        out = (Assignment * n)()
        batches = (Batch * max(n, 1))()
        cnt = C.c_uint32(0)
        ok = self.lib.ref_group_tokens_by_expert(a, n, out, batches, max(n, 1), C.byref(cnt))
        return ok, out, batches, cnt.value


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def metadata_json(top_k: int, norm_topk: bool = False, sigmoid: bool = False,
                  routed_scale: float = 1.0, n_group: int = 0, topk_group: int = 0,
                  block: Optional[Block] = None) -> str:
    """GGUF metadata keys the reference router reads
    (generation_router.cpp.inc:361-558), plus the block's activation and
    norm style."""
    parts = [f'"num_experts_per_tok":{int(top_k)}', f'"norm_topk_prob":{"true" if norm_topk else "false"}']
    if block is not None:
        parts += block.metadata()
    if sigmoid:
        parts.append('"scoring_func":"sigmoid"')
        if routed_scale != 1.0:
            parts.append(f'"routed_scaling_factor":{routed_scale!r}')
    if n_group:
        parts.append(f'"n_group":{int(n_group)}')
        parts.append(f'"topk_group":{int(topk_group)}')
    return "{" + ",".join(parts) + "}"
