"""ctypes binding of libmoe_b200.so (the C ABI in include/moe_b200.h).

This is the Python face of the product path: every call goes straight to
the CUDA library.  There is no CPU fallback -- constructing an Engine fails
loudly when the library or a B200 is missing.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmoe_b200.so"
HEADER = HERE.parent / "include" / "moe_b200.h"
ERR_LEN = 160
EP_UID_BYTES = 128

SCORE_SOFTMAX, SCORE_SIGMOID = 0, 1
ACT_SILU, ACT_GELU_ERF, ACT_GELU_TANH = 0, 1, 2
GEMM_BLOCKSCALED, GEMM_SIMT, GEMM_TMEM_DECODE, GEMM_MXF4_FAST = 0, 1, 2, 3
GEMM_TCGEN05 = GEMM_BLOCKSCALED
PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2
BUF_LOGITS, BUF_SCORES, BUF_GROUP_COUNT, BUF_GROUP_OFFSET, BUF_ROW_TOKEN, BUF_XPERM, BUF_HPERM, BUF_YPERM = range(8)


class InitT(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_layers", C.c_uint32)]


class LayerCfg(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("experts", C.c_uint32),
                ("top_k", C.c_uint32), ("layer", C.c_int32), ("score_func", C.c_int32),
                ("norm_topk", C.c_int32), ("routed_scale", C.c_float), ("use_shared", C.c_int32),
                ("gemm_path", C.c_int32), ("n_group", C.c_uint32), ("topk_group", C.c_uint32),
                ("activation", C.c_int32), ("norm_unit_offset", C.c_int32), ("norm_eps", C.c_float),
                ("skip_missing", C.c_int32)]


class BlockTensors(C.Structure):
    _fields_ = [("pre_norm2", C.c_void_p), ("post_norm1", C.c_void_p), ("post_norm2", C.c_void_p),
                ("post_norm", C.c_void_p), ("down_scale", C.c_void_p), ("down_scale_count", C.c_uint64),
                ("shared_gate_inp", C.c_void_p), ("router_scale", C.c_void_p), ("router_scale_count", C.c_uint64)]


class Assignment(C.Structure):
    _fields_ = [("token_index", C.c_uint32), ("layer", C.c_uint32), ("expert", C.c_uint32),
                ("router_score", C.c_float)]


class Batch(C.Structure):
    _fields_ = [("layer", C.c_uint32), ("expert", C.c_uint32), ("first_sorted_index", C.c_uint32),
                ("token_count", C.c_uint32)]


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    return re.findall(r"MOE_B200_API\s+[\w\*\s]+?\b(moe_b200_\w+)\s*\(", HEADER.read_text())


_lib = None


def load(path: Path = LIB_PATH) -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not path.exists():
        raise RuntimeError(f"{path} is missing: build it with `python storage.llm_b200/build.py`")
    lib = C.CDLL(str(path))
    vp, cp = C.c_void_p, C.c_char_p
    lib.moe_b200_create.restype = vp
    lib.moe_b200_create.argtypes = [C.POINTER(InitT), cp]
    lib.moe_b200_destroy.argtypes = [vp]
    lib.moe_b200_upload_router.restype = C.c_int
    lib.moe_b200_upload_router.argtypes = [vp, C.c_int32, vp, C.c_uint32, C.c_uint32, C.c_int32, cp]
    lib.moe_b200_upload_expert.restype = C.c_int
    lib.moe_b200_upload_expert.argtypes = [vp, C.c_int32, C.c_int32, vp, C.c_uint64, vp, C.c_uint64, vp,
                                           C.c_uint64, C.c_uint32, C.c_uint32, C.c_int32, cp]
    lib.moe_b200_expert_record_bytes.restype = C.c_uint64
    lib.moe_b200_expert_record_bytes.argtypes = [C.c_uint32, C.c_uint32]
    lib.moe_b200_export_expert.restype = C.c_int
    lib.moe_b200_export_expert.argtypes = [vp, C.c_int32, C.c_int32, vp, C.c_uint64, C.c_int32, cp]
    lib.moe_b200_import_expert.restype = C.c_int
    lib.moe_b200_import_expert.argtypes = [vp, C.c_int32, C.c_int32, vp, C.c_uint64, C.c_uint32, C.c_uint32,
                                           C.c_int32, cp]
    lib.moe_b200_source_key.restype = C.c_uint64
    lib.moe_b200_source_key.argtypes = [vp, C.c_uint64, vp, C.c_uint64, vp, C.c_uint64]
    lib.moe_b200_expert_cache_open.restype = vp
    lib.moe_b200_expert_cache_open.argtypes = [C.c_char_p, cp]
    lib.moe_b200_expert_cache_close.argtypes = [vp]
    lib.moe_b200_expert_cache_info.restype = C.c_int
    lib.moe_b200_expert_cache_info.argtypes = [vp, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                               C.POINTER(C.c_uint64), C.POINTER(C.c_uint32)]
    lib.moe_b200_expert_cache_record.restype = vp
    lib.moe_b200_expert_cache_record.argtypes = [vp, C.c_int32, C.c_int32, C.c_uint64, C.c_int32, cp]
    lib.moe_b200_layer_forward.restype = C.c_int
    lib.moe_b200_layer_forward.argtypes = [vp, C.POINTER(LayerCfg), vp, C.c_uint32, vp, vp, vp, vp, vp, vp, cp]
    lib.moe_b200_layer_forward_host.restype = C.c_int
    lib.moe_b200_layer_forward_host.argtypes = [vp, C.POINTER(LayerCfg), vp, C.c_uint32, vp, vp, vp, vp, vp, cp]
    lib.moe_b200_upload_block.restype = C.c_int
    lib.moe_b200_upload_block.argtypes = [vp, C.c_int32, C.POINTER(BlockTensors), C.c_int32, cp]
    lib.moe_b200_block_forward.restype = C.c_int
    lib.moe_b200_block_forward.argtypes = [vp, C.POINTER(LayerCfg), vp, vp, C.c_uint32, vp, vp, vp, vp, vp, cp]
    lib.moe_b200_block_forward_host.restype = C.c_int
    lib.moe_b200_block_forward_host.argtypes = [vp, C.POINTER(LayerCfg), vp, vp, C.c_uint32, vp, vp, vp, vp, cp]
    lib.moe_b200_sync.restype = C.c_int
    lib.moe_b200_sync.argtypes = [vp, vp, cp]
    lib.moe_b200_run_expert_triplet_f32.restype = C.c_int
    lib.moe_b200_run_expert_triplet_f32.argtypes = [vp, C.c_int, C.c_int, vp, C.c_uint32, vp, vp, C.c_uint32,
                                                    vp, C.c_uint32]
    lib.moe_b200_group_tokens_by_expert.restype = C.c_int
    lib.moe_b200_group_tokens_by_expert.argtypes = [C.POINTER(Assignment), C.c_uint32, C.POINTER(Assignment),
                                                    C.POINTER(Batch), C.c_uint32, C.POINTER(C.c_uint32)]
    lib.moe_b200_group_tokens_by_expert_noalloc.restype = C.c_int
    lib.moe_b200_group_tokens_by_expert_noalloc.argtypes = [C.POINTER(Assignment), C.c_uint32,
                                                            C.POINTER(Assignment), C.POINTER(Batch), C.c_uint32,
                                                            C.POINTER(C.c_uint32), cp]
    lib.moe_b200_debug_dequant.restype = C.c_int
    lib.moe_b200_debug_dequant.argtypes = [vp, C.c_int32, C.c_int32, C.c_int32, vp, C.c_uint64, cp]
    lib.moe_b200_debug_read.restype = C.c_int
    lib.moe_b200_debug_read.argtypes = [vp, C.c_int32, vp, C.c_uint64, cp]
    lib.moe_b200_profile_enable.restype = C.c_int
    lib.moe_b200_profile_enable.argtypes = [vp, C.c_uint32, cp]
    lib.moe_b200_profile_read.restype = C.c_int
    lib.moe_b200_profile_read.argtypes = [vp, C.POINTER(C.c_float), C.POINTER(C.c_uint32), cp]
    lib.moe_b200_last_launch_count.restype = C.c_uint32
    lib.moe_b200_last_launch_count.argtypes = [vp]
    lib.moe_b200_ep_unique_id.restype = C.c_int
    lib.moe_b200_ep_unique_id.argtypes = [vp, cp]
    lib.moe_b200_ep_init.restype = C.c_int
    lib.moe_b200_ep_init.argtypes = [vp, C.c_int, C.c_int, vp, cp]
    lib.moe_b200_ep_local_experts.restype = C.c_int
    lib.moe_b200_ep_local_experts.argtypes = [vp, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), cp]
    lib.moe_b200_ep_layer_forward.restype = C.c_int
    lib.moe_b200_ep_layer_forward.argtypes = [vp, C.POINTER(LayerCfg), vp, C.c_uint32, vp, vp, vp, vp, vp, cp]
    lib.moe_b200_ep_layer_forward_host.restype = C.c_int
    lib.moe_b200_ep_layer_forward_host.argtypes = [vp, C.POINTER(LayerCfg), vp, C.c_uint32, vp, vp, vp, vp, cp]
    lib.moe_b200_ep_set_placement.restype = C.c_int
    lib.moe_b200_ep_set_placement.argtypes = [vp, C.c_uint32, vp, vp, cp]
    lib.moe_b200_ep_local_expert_list.restype = C.c_int
    lib.moe_b200_ep_local_expert_list.argtypes = [vp, C.c_uint32, vp, C.c_uint32, C.POINTER(C.c_uint32), cp]
    lib.moe_b200_ep_last_counts.restype = C.c_int
    lib.moe_b200_ep_last_counts.argtypes = [vp, vp, vp, cp]
    _lib = lib
    return lib


def _ptr(a) -> Optional[int]:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"]
        return a.ctypes.data
    return int(a.data_ptr())  # torch tensor (device or pinned host)


class MoEError(RuntimeError):
    pass


class Engine:
    """One engine per CUDA device (moe_b200_create)."""

    def __init__(self, device: int = 0, max_layers: int = 1):
        self.lib = load()
        self.err = C.create_string_buffer(ERR_LEN)
        init = InitT(device, max_layers)
        self.h = self.lib.moe_b200_create(C.byref(init), self.err)
        if not self.h:
            raise MoEError(self.err.value.decode())

    def _check(self, ok: int):
        if not ok:
            raise MoEError(self.err.value.decode())

    def close(self):
        if self.h:
            self.lib.moe_b200_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights ----------------------------------------------------------
    def upload_router(self, layer: int, router, experts: int, hidden: int, on_device: bool = False):
        self._check(self.lib.moe_b200_upload_router(self.h, layer, _ptr(router), experts, hidden,
                                                    int(on_device), self.err))

    def upload_expert(self, layer: int, expert: int, gate, up, down, hidden: int, intermediate: int,
                      on_device: bool = False):
        nb = lambda a: a.nbytes if isinstance(a, np.ndarray) else a.numel() * a.element_size()
        self._check(self.lib.moe_b200_upload_expert(self.h, layer, expert, _ptr(gate), nb(gate), _ptr(up), nb(up),
                                                    _ptr(down), nb(down), hidden, intermediate, int(on_device),
                                                    self.err))

    def record_bytes(self, hidden: int, intermediate: int) -> int:
        """Bytes of one repacked-expert record for experts of this shape."""
        return int(self.lib.moe_b200_expert_record_bytes(hidden, intermediate))

    def export_expert(self, layer: int, expert: int, hidden: int, intermediate: int) -> np.ndarray:
        """A resident expert's repacked record (expert -1: the shared expert) as host bytes."""
        out = np.empty(self.record_bytes(hidden, intermediate), np.uint8)
        self._check(self.lib.moe_b200_export_expert(self.h, layer, expert, _ptr(out), out.nbytes, 0, self.err))
        return out

    def import_expert(self, layer: int, expert: int, record, hidden: int, intermediate: int,
                      on_device: bool = False):
        """Installs a repacked record (host numpy bytes, or a device tensor with
        on_device) as upload_expert would have left the expert, without the repack."""
        nb = record.nbytes if isinstance(record, np.ndarray) else record.numel() * record.element_size()
        self._check(self.lib.moe_b200_import_expert(self.h, layer, expert, _ptr(record), nb, hidden, intermediate,
                                                    int(on_device), self.err))

    def upload_layer(self, li, layer: int = 0):
        """Uploads a synth.LayerInputs (host numpy GGUF bytes)."""
        s = li.shape
        self.upload_router(layer, np.ascontiguousarray(li.router), s.experts, s.hidden)
        for e in range(s.experts):
            self.upload_expert(layer, e, np.ascontiguousarray(li.gate[e]), np.ascontiguousarray(li.up[e]),
                               np.ascontiguousarray(li.down[e]), s.hidden, s.intermediate)
        if li.shared_gate is not None:
            self.upload_expert(layer, -1, np.ascontiguousarray(li.shared_gate), np.ascontiguousarray(li.shared_up),
                               np.ascontiguousarray(li.shared_down), s.hidden, s.intermediate)

    @staticmethod
    def cfg(shape, layer: int = 0, gemm_path: int = GEMM_TCGEN05, score_func: int = SCORE_SOFTMAX,
            norm_topk: Optional[bool] = None, routed_scale: float = 1.0, use_shared: Optional[bool] = None,
            n_group: int = 0, topk_group: int = 0, activation: int = ACT_SILU, norm_unit_offset: bool = False,
            norm_eps: float = 0.0, skip_missing: bool = False):
        nt = shape.norm_topk if norm_topk is None else norm_topk
        us = shape.shared if use_shared is None else use_shared
        return LayerCfg(shape.hidden, shape.intermediate, shape.experts, shape.top_k, layer, score_func, int(nt),
                        routed_scale, int(us), gemm_path, n_group, topk_group, activation, int(norm_unit_offset),
                        norm_eps, int(skip_missing))

    def upload_block(self, layer: int, pre_norm2=None, post_norm1=None, post_norm2=None, post_norm=None,
                     down_scale=None, shared_gate_inp=None, router_scale=None):
        """The block tensors of a layer from host numpy arrays (None = absent)."""
        keep = {}

        def arr(name, a, dtype):
            if a is None:
                return None
            keep[name] = np.ascontiguousarray(a, dtype=dtype)
            return keep[name].ctypes.data

        t = BlockTensors(arr("pn2", pre_norm2, np.float32), arr("n1", post_norm1, np.float32),
                         arr("n2", post_norm2, np.float32), arr("n", post_norm, np.float32),
                         arr("ds", down_scale, np.float32), 0 if down_scale is None else int(np.size(down_scale)),
                         arr("sg", shared_gate_inp, np.uint16), arr("rs", router_scale, np.float32),
                         0 if router_scale is None else int(np.size(router_scale)))
        self._check(self.lib.moe_b200_upload_block(self.h, layer, C.byref(t), 0, self.err))

    def clear_block(self, layer: int):
        self._check(self.lib.moe_b200_upload_block(self.h, layer, None, 0, self.err))

    def block_forward_host(self, cfg: LayerCfg, x: np.ndarray, hidden: Optional[np.ndarray] = None):
        T = x.shape[0]
        H, K = cfg.hidden, cfg.top_k
        y = np.zeros((T, H), np.uint16)
        yf = np.zeros((T, H), np.float32)
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        x = np.ascontiguousarray(x, dtype=np.uint16)
        hid = None if hidden is None else np.ascontiguousarray(hidden, dtype=np.float32)
        self._check(self.lib.moe_b200_block_forward_host(self.h, C.byref(cfg), _ptr(x), _ptr(hid), T, _ptr(y),
                                                         _ptr(yf), _ptr(ids), _ptr(w), self.err))
        return dict(y_bf16=y, y_f32=yf, ids=ids, w=w)

    # -- forward ----------------------------------------------------------
    def forward(self, cfg: LayerCfg, x, tokens: int, y_bf16=None, y_f32=None, ids=None, w=None, perm=None,
                stream: int = 0):
        """Device-pointer forward (torch CUDA tensors); enqueued on `stream`."""
        self._check(self.lib.moe_b200_layer_forward(self.h, C.byref(cfg), _ptr(x), tokens, _ptr(y_bf16),
                                                    _ptr(y_f32), _ptr(ids), _ptr(w), _ptr(perm), stream,
                                                    self.err))

    def forward_host(self, cfg: LayerCfg, x: np.ndarray, want_f32: bool = True, want_perm: bool = True):
        """want_perm=False leaves the permutation out, which lets large
        batches overlap their copies with the router and the combine."""
        T = x.shape[0]
        H, K = cfg.hidden, cfg.top_k
        y = np.zeros((T, H), np.uint16)
        yf = np.zeros((T, H), np.float32) if want_f32 else None
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        perm = np.zeros(T * K, np.uint32) if want_perm else None
        x = np.ascontiguousarray(x, dtype=np.uint16)
        self._check(self.lib.moe_b200_layer_forward_host(self.h, C.byref(cfg), _ptr(x), T, _ptr(y), _ptr(yf),
                                                         _ptr(ids), _ptr(w), _ptr(perm), self.err))
        return dict(y_bf16=y, y_f32=yf, ids=ids, w=w, perm=perm)

    def sync(self, stream: int = 0):
        self._check(self.lib.moe_b200_sync(self.h, stream, self.err))

    # -- expert parallelism ------------------------------------------------
    @staticmethod
    def ep_unique_id() -> bytes:
        lib = load()
        buf = (C.c_uint8 * EP_UID_BYTES)()
        err = C.create_string_buffer(ERR_LEN)
        if not lib.moe_b200_ep_unique_id(buf, err):
            raise MoEError(err.value.decode(errors="replace"))
        return bytes(buf)

    def ep_init(self, rank: int, world: int, uid: bytes):
        buf = (C.c_uint8 * EP_UID_BYTES).from_buffer_copy(uid)
        self._check(self.lib.moe_b200_ep_init(self.h, rank, world, buf, self.err))

    def ep_local_experts(self, experts: int):
        first, count = C.c_uint32(0), C.c_uint32(0)
        self._check(self.lib.moe_b200_ep_local_experts(self.h, experts, C.byref(first), C.byref(count), self.err))
        return first.value, count.value

    def ep_set_placement(self, replicas):
        """replicas[e] = list of ranks holding expert e (the same on every rank)."""
        cnt = np.array([len(r) for r in replicas], np.uint32)
        ranks = np.array([q for r in replicas for q in r], np.uint32)
        self._check(self.lib.moe_b200_ep_set_placement(self.h, len(replicas), _ptr(cnt), _ptr(ranks), self.err))

    def ep_local_expert_list(self, experts: int):
        out = np.zeros(experts, np.uint32)
        cnt = C.c_uint32(0)
        self._check(self.lib.moe_b200_ep_local_expert_list(self.h, experts, _ptr(out), experts, C.byref(cnt),
                                                           self.err))
        return [int(e) for e in out[:cnt.value]]

    def upload_layer_ep(self, li, layer: int = 0):
        """Router, this rank's experts (current placement) and the shared expert."""
        s = li.shape
        self.upload_router(layer, np.ascontiguousarray(li.router), s.experts, s.hidden)
        for e in self.ep_local_expert_list(s.experts):
            self.upload_expert(layer, e, np.ascontiguousarray(li.gate[e]), np.ascontiguousarray(li.up[e]),
                               np.ascontiguousarray(li.down[e]), s.hidden, s.intermediate)
        if li.shared_gate is not None:
            self.upload_expert(layer, -1, np.ascontiguousarray(li.shared_gate), np.ascontiguousarray(li.shared_up),
                               np.ascontiguousarray(li.shared_down), s.hidden, s.intermediate)

    def ep_forward(self, cfg: LayerCfg, x, tokens: int, y_bf16=None, y_f32=None, ids=None, w=None, stream: int = 0):
        self._check(self.lib.moe_b200_ep_layer_forward(self.h, C.byref(cfg), _ptr(x), tokens, _ptr(y_bf16),
                                                       _ptr(y_f32), _ptr(ids), _ptr(w), stream, self.err))

    def ep_forward_host(self, cfg: LayerCfg, x: np.ndarray, want_f32: bool = True):
        T = x.shape[0]
        H, K = cfg.hidden, cfg.top_k
        y = np.zeros((T, H), np.uint16)
        yf = np.zeros((T, H), np.float32) if want_f32 else None
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        x = np.ascontiguousarray(x, dtype=np.uint16)
        self._check(self.lib.moe_b200_ep_layer_forward_host(self.h, C.byref(cfg), _ptr(x), T, _ptr(y), _ptr(yf),
                                                            _ptr(ids), _ptr(w), self.err))
        return dict(y_bf16=y, y_f32=yf, ids=ids, w=w)

    def ep_last_counts(self, world: int):
        sent = np.zeros(world, np.uint32)
        recv = np.zeros(world, np.uint32)
        self._check(self.lib.moe_b200_ep_last_counts(self.h, _ptr(sent), _ptr(recv), self.err))
        return sent, recv

    STAGES = ("router", "permute", "gather", "gate_up", "down", "combine")

    def profile_enable(self, max_calls: int):
        self._check(self.lib.moe_b200_profile_enable(self.h, max_calls, self.err))

    def profile_read(self):
        ms = (C.c_float * len(self.STAGES))()
        calls = C.c_uint32(0)
        self._check(self.lib.moe_b200_profile_read(self.h, ms, C.byref(calls), self.err))
        return dict(zip(self.STAGES, [float(v) for v in ms])), calls.value

    def launches(self) -> int:
        return int(self.lib.moe_b200_last_launch_count(self.h))

    # -- other entry points ----------------------------------------------
    def expert_triplet(self, layer: int, expert: int, hidden: np.ndarray, intermediate: int):
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        H = hidden.shape[0]
        g = np.zeros(intermediate, np.float32)
        u = np.zeros(intermediate, np.float32)
        out = np.zeros(H, np.float32)
        ok = self.lib.moe_b200_run_expert_triplet_f32(self.h, layer, expert, _ptr(hidden), H, _ptr(g), _ptr(u),
                                                      intermediate, _ptr(out), H)
        if not ok:
            raise MoEError("moe_b200_run_expert_triplet_f32 failed")
        return g, u, out

    def dequant(self, layer: int, expert: int, proj: int, rows: int, cols: int) -> np.ndarray:
        out = np.zeros((rows, cols), np.uint16)
        self._check(self.lib.moe_b200_debug_dequant(self.h, layer, expert, proj, _ptr(out), out.size, self.err))
        return out

    def read(self, which: int, shape, dtype) -> np.ndarray:
        out = np.zeros(shape, dtype)
        self._check(self.lib.moe_b200_debug_read(self.h, which, _ptr(out), out.nbytes, self.err))
        return out


def group_tokens_by_expert(token, expert, score=None, layer=None, max_batches: Optional[int] = None):
    """moe_b200_group_tokens_by_expert on the current CUDA device."""
    lib = load()
    n = len(token)
    a = (Assignment * max(n, 1))()
    for i in range(n):
        a[i] = Assignment(int(token[i]), 0 if layer is None else int(layer[i]), int(expert[i]),
                          0.0 if score is None else float(score[i]))
    out = (Assignment * max(n, 1))()
    mb = n if max_batches is None else max_batches
    batches = (Batch * max(mb, 1))()
    cnt = C.c_uint32(0)
    ok = lib.moe_b200_group_tokens_by_expert(a, n, out, batches, mb, C.byref(cnt))
    return ok, out, batches, cnt.value
