"""Seeded synthetic frames with the shapes and value distributions of the benchmark configurations.

The reference measures on no public dataset; every input here is synthetic:
  Q/K/V ~ N(0,1) rounded to the storage dtype, RMSNorm weights ~ N(1, 0.1), cached K/V ~ N(0,1),
  active mask i.i.d. Bernoulli(p) per image token (or a union of rectangles), text tokens always
  executed and updated (mask 2). Position ids: image (0, h, w) on the patch grid, text (0, 0, 0)
  for the 3-axis 16/56/56 layout; the 4-axis Klein layout uses (0, h, w, 0) / (0, 0, 0, l).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    grid_h: int             # image tokens = grid_h * grid_w
    grid_w: int
    n_text: int
    n_heads: int = 24
    head_dim: int = 128
    dtype: str = "bf16"
    active: float = 0.25
    pattern: str = "bernoulli"     # "bernoulli" | "rects"
    rope_axes: tuple = (16, 56, 56)
    rope_theta: float = 10000.0

    @property
    def n_image(self) -> int:
        return self.grid_h * self.grid_w

    @property
    def n_tokens(self) -> int:
        return self.n_text + self.n_image


# Benchmark configurations (frame side / 16 = patch grid side).
C1 = Workload("c1_512px_p25_f16", 32, 32, 512, dtype="f16", active=0.25)
C2 = Workload("c2_1024px_p25_bf16", 64, 64, 512, active=0.25)
C3 = Workload("c3_1024px_rects_bf16", 64, 64, 512, pattern="rects", active=0.20)
C4 = Workload("c4_768px_p25_bf16", 48, 48, 512, active=0.25)
C5 = Workload("c5_2048px_p15_bf16", 128, 128, 512, active=0.15)
KLEIN = Workload("klein_4axis_theta2000", 32, 32, 256, dtype="f16", rope_axes=(32, 32, 32, 32),
                 rope_theta=2000.0)

BY_NAME = {w.name: w for w in (C1, C2, C3, C4, C5, KLEIN)}


def with_active(w: Workload, p: float) -> Workload:
    return Workload(f"{w.name.split('_p')[0]}_p{int(round(p * 100))}", w.grid_h, w.grid_w, w.n_text,
                    w.n_heads, w.head_dim, w.dtype, p, w.pattern, w.rope_axes, w.rope_theta)


def positions(w: Workload) -> np.ndarray:
    """int32 [N, n_axes] position ids, text rows first."""
    n_axes = len(w.rope_axes)
    pos = np.zeros((w.n_tokens, n_axes), dtype=np.int32)
    hh, ww = np.meshgrid(np.arange(w.grid_h), np.arange(w.grid_w), indexing="ij")
    img = pos[w.n_text:]
    if n_axes >= 3:
        img[:, 1] = hh.reshape(-1)
        img[:, 2] = ww.reshape(-1)
    if n_axes == 4:
        pos[: w.n_text, 3] = np.arange(w.n_text)
    return pos


def make_mask(w: Workload, rng: np.random.Generator, p: float | None = None) -> np.ndarray:
    """int32 [N] change mask: text = 2, image 2 where edited else 0."""
    p = w.active if p is None else p
    mask = np.zeros(w.n_tokens, dtype=np.int32)
    mask[: w.n_text] = 2
    if w.pattern == "rects":
        img = np.zeros((w.grid_h, w.grid_w), dtype=bool)
        target = p * w.n_image
        while img.sum() < target:
            for _ in range(int(rng.integers(1, 5))):
                hs, ws = int(rng.integers(8, 41)), int(rng.integers(8, 41))
                y0, x0 = int(rng.integers(0, max(1, w.grid_h - hs + 1))), int(rng.integers(0, max(1, w.grid_w - ws + 1)))
                img[y0:y0 + hs, x0:x0 + ws] = True
                if img.sum() >= target:
                    break
        mask[w.n_text:] = np.where(img.reshape(-1), 2, 0)
    else:
        mask[w.n_text:] = np.where(rng.random(w.n_image) < p, 2, 0)
    return mask


def round_storage(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> storage dtype (round to nearest even) -> fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = np.ascontiguousarray(x).view(np.uint32)
        r = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
        return r.astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


def make_frame(w: Workload, seed: int = 0, p: float | None = None) -> dict:
    """Host (numpy, fp32 values exactly representable in the storage dtype) frame inputs."""
    rng = np.random.default_rng(seed)
    N, C = w.n_tokens, w.n_heads * w.head_dim
    f = lambda shape, mu=0.0, sd=1.0: rng.normal(mu, sd, size=shape).astype(np.float32)
    out = {
        "q": round_storage(f((N, C)), w.dtype),
        "k": round_storage(f((N, C)), w.dtype),
        "v": round_storage(f((N, C)), w.dtype),
        "cache_k": round_storage(f((N, C)), w.dtype),
        "cache_v": round_storage(f((N, C)), w.dtype),
        "out": round_storage(f((N, C)), w.dtype),
        "norm_q": f((w.head_dim,), 1.0, 0.1),
        "norm_k": f((w.head_dim,), 1.0, 0.1),
        "mask": make_mask(w, rng, p),
        "pos": positions(w),
    }
    return out
