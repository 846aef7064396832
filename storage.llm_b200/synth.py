"""Seeded synthetic inputs for the MoE expert-FFN layer.

There is no public dataset for this path; every configuration is synthetic
and generated the same way for the CUDA path, the C oracle and the compiled
reference:

* router weight ``ffn_gate_inp.weight``: bf16 ``[E x H]`` ~ N(0, 0.02);
* expert weights: GGUF MXFP4 bytes (the reference's on-disk layout,
  tensor_layout.cpp.inc:174-176): per row, ``ceil(K/32)`` blocks of 17 bytes
  = one E8M0 scale byte then 16 code bytes, element j in the low nibble of
  byte j and element j+16 in the high nibble
  (tensor_dot_cpu_kernels.cpp.inc:595-599).  Codes are uniform over the 16
  E2M1 codes and every scale byte is 120 (2^-7), giving a weight std of
  2.926 * 2^-7 ~= 0.0229, the power of two closest to the 0.02 target;
* activations: bf16 ~ N(mu, 1).  ``mu = 0`` except for the skewed
  configurations.  The reference router has no bias term, so a popularity
  skew is realised as a token-independent mean shift ``mu`` with
  ``W mu = b`` (minimum-norm least squares), ``b`` calibrated so that the
  realised top-k histogram follows the configuration's target popularity.
"""
from __future__ import annotations

import dataclasses
import hashlib
from typing import Optional

import numpy as np

MXFP4_BLOCK = 32
MXFP4_BLOCK_BYTES = 17
SCALE_BYTE = 120  # E8M0 2^(120-127)


@dataclasses.dataclass
class LayerShape:
    name: str
    hidden: int
    intermediate: int
    experts: int
    top_k: int
    tokens: int
    shared: bool = False
    skew: Optional[str] = None  # None | "zipf1.1" | "hot10_40"
    norm_topk: bool = False


# The five configurations of the headline benchmark, at their full sizes.
CONFIGS = {
    0: LayerShape("c0_h1024_e8_k2_i2816", 1024, 2816, 8, 2, 64),
    1: LayerShape("c1_h2880_e32_k4_i2880_decode", 2880, 2880, 32, 4, 256, skew="zipf1.1"),
    2: LayerShape("c2_h2880_e128_k4_i2880_prefill", 2880, 2880, 128, 4, 0),
    3: LayerShape("c3_h2048_e128_k8_i768", 2048, 768, 128, 8, 4096, skew="hot10_40"),
    4: LayerShape("c4_h7168_e256_k8_i2048_shared", 7168, 2048, 256, 8, 16384, shared=True),
}
DECODE_SWEEP = (1, 8, 32, 128, 256)


def prefill_lengths(seed: int = 2) -> list[int]:
    """Config 2: 8 packed sequences with lengths uniform in [128, 2048]."""
    rng = np.random.default_rng(seed + 1000)
    return [int(v) for v in rng.integers(128, 2049, size=8)]


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def mxfp4_row_bytes(cols: int) -> int:
    return (cols + MXFP4_BLOCK - 1) // MXFP4_BLOCK * MXFP4_BLOCK_BYTES


def gen_mxfp4(rng: np.random.Generator, lead: tuple, rows: int, cols: int,
              scale_byte: int = SCALE_BYTE) -> np.ndarray:
    """GGUF MXFP4 bytes of shape lead + (rows, row_bytes)."""
    nblk = (cols + MXFP4_BLOCK - 1) // MXFP4_BLOCK
    out = np.empty(lead + (rows, nblk, MXFP4_BLOCK_BYTES), dtype=np.uint8)
    out[..., 0] = scale_byte
    # one leading index (expert) at a time: the same bytes as one draw of the
    # whole array (each chunk is a multiple of 4 bytes, so the generator's
    # 32-bit words split evenly), without a second full-size temporary
    flat = out.reshape((-1, rows, nblk, MXFP4_BLOCK_BYTES))
    for i in range(flat.shape[0]):
        flat[i, ..., 1:] = rng.integers(0, 256, size=(rows, nblk, 16), dtype=np.uint8)
    tail = cols % MXFP4_BLOCK
    if tail:
        # Elements past `cols` in the last block are never read by the
        # reference; keep them zero so every consumer sees identical bytes.
        codes = out[..., nblk - 1, 1:]
        for j in range(16):
            keep_lo = j < tail
            keep_hi = j + 16 < tail
            mask = (0x0F if keep_lo else 0) | (0xF0 if keep_hi else 0)
            codes[..., j] &= mask
    return out.reshape(lead + (rows, nblk * MXFP4_BLOCK_BYTES))


def jitter_scales(packed: np.ndarray, rng: np.random.Generator, spread: int, up: int = 0) -> np.ndarray:
    """Copy of GGUF MXFP4 bytes with every block's E8M0 scale byte moved by a
    seeded offset in [-spread, up] (real checkpoints vary their scales per
    32-element block; the default generator uses one scale everywhere)."""
    shp = packed.shape
    blk = packed.reshape(shp[:-1] + (shp[-1] // MXFP4_BLOCK_BYTES, MXFP4_BLOCK_BYTES)).copy()
    off = rng.integers(-spread, up + 1, size=blk.shape[:-1])
    blk[..., 0] = np.clip(blk[..., 0].astype(np.int64) + off, 0, 254).astype(np.uint8)
    return blk.reshape(shp)


def target_popularity(skew: str, experts: int, rng: np.random.Generator) -> np.ndarray:
    if skew == "zipf1.1":
        ranks = np.arange(1, experts + 1, dtype=np.float64)
        p = ranks ** -1.1
    elif skew == "hot10_40":
        hot = max(1, int(round(0.1 * experts)))
        p = np.full(experts, 0.6 / (experts - hot))
        p[:hot] = 0.4 / hot
    else:
        raise ValueError(skew)
    p = p / p.sum()
    return p[rng.permutation(experts)]


def _topk_hist(logits: np.ndarray, k: int) -> np.ndarray:
    idx = np.argpartition(-logits, k - 1, axis=1)[:, :k]
    return np.bincount(idx.ravel(), minlength=logits.shape[1]).astype(np.float64)


def calibrate_bias(wf: np.ndarray, k: int, target: np.ndarray, rng: np.random.Generator,
                   sample: int = 4096, iters: int = 60) -> np.ndarray:
    """Logit bias b whose realised top-k histogram follows `target`."""
    e, h = wf.shape
    noise = rng.standard_normal((sample, h)).astype(np.float32) @ wf.T.astype(np.float32)
    noise = noise.astype(np.float64)
    b = np.log(target) - np.log(target).mean()
    want = target * sample * k
    for _ in range(iters):
        hist = _topk_hist(noise + b, k)
        b += 0.5 * (np.log(want + 1.0) - np.log(hist + 1.0))
        b -= b.mean()
    return b


@dataclasses.dataclass
class LayerInputs:
    shape: LayerShape
    router: np.ndarray          # uint16 [E, H]
    gate: np.ndarray            # uint8 [E, I, rowbytes(H)]
    up: np.ndarray              # uint8 [E, I, rowbytes(H)]
    down: np.ndarray            # uint8 [E, H, rowbytes(I)]
    x: np.ndarray               # uint16 [T, H]
    shared_gate: Optional[np.ndarray] = None
    shared_up: Optional[np.ndarray] = None
    shared_down: Optional[np.ndarray] = None
    mu: Optional[np.ndarray] = None

    def digest(self) -> str:
        h = hashlib.sha256()
        for a in (self.router, self.gate, self.up, self.down, self.x,
                  self.shared_gate, self.shared_up, self.shared_down):
            if a is not None:
                h.update(np.ascontiguousarray(a).reshape(-1).view(np.uint8))
        return h.hexdigest()


def gen_weights(shape: LayerShape, seed: int):
    rng = np.random.default_rng([seed, 1])
    H, I, E = shape.hidden, shape.intermediate, shape.experts
    router = f32_to_bf16_bits(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02))
    gate = gen_mxfp4(rng, (E,), I, H)
    up = gen_mxfp4(rng, (E,), I, H)
    down = gen_mxfp4(rng, (E,), H, I)
    shared = None
    if shape.shared:
        shared = (gen_mxfp4(rng, (), I, H), gen_mxfp4(rng, (), I, H), gen_mxfp4(rng, (), H, I))
    return router, gate, up, down, shared


def gen_mean_shift(shape: LayerShape, router: np.ndarray, seed: int) -> Optional[np.ndarray]:
    if not shape.skew:
        return None
    rng = np.random.default_rng([seed, 2])
    wf = bf16_bits_to_f32(router).astype(np.float64)
    target = target_popularity(shape.skew, shape.experts, rng)
    b = calibrate_bias(wf, shape.top_k, target, rng)
    mu, *_ = np.linalg.lstsq(wf, b, rcond=None)
    return mu.astype(np.float32)


def gen_tokens(shape: LayerShape, tokens: int, seed: int, mu: Optional[np.ndarray]) -> np.ndarray:
    rng = np.random.default_rng([seed, 3, tokens])
    x = rng.standard_normal((tokens, shape.hidden), dtype=np.float32)
    if mu is not None:
        x += mu[None, :]
    return f32_to_bf16_bits(x)


def make_layer(shape: LayerShape, seed: int = 0, tokens: Optional[int] = None) -> LayerInputs:
    router, gate, up, down, shared = gen_weights(shape, seed)
    mu = gen_mean_shift(shape, router, seed)
    t = shape.tokens if tokens is None else tokens
    if t == 0:
        t = sum(prefill_lengths(seed))
    x = gen_tokens(shape, t, seed, mu)
    li = LayerInputs(shape, router, gate, up, down, x, mu=mu)
    if shared is not None:
        li.shared_gate, li.shared_up, li.shared_down = shared
    return li


def small_shape(name="mini", hidden=64, intermediate=96, experts=8, top_k=2, tokens=16,
                shared=False, skew=None, norm_topk=False) -> LayerShape:
    return LayerShape(name, hidden, intermediate, experts, top_k, tokens, shared, skew, norm_topk)
