"""Seeded synthetic workloads of the five sampler configurations.

No public dataset or checkpoint is involved: the configurations in
BASELINE.json define the logit distributions, and these generators reproduce
them from a seed (numpy Philox4x32-10 streams keyed by (seed, step)).  Draws u
are 53-bit doubles in [0, 1), the value the reference's `Random` supplies
(src/Gemma4.Model.pas:2726, 2813).

  C1  one row, V=262144 fp32 ~ N(0, 3^2) with 16 distinct random ids +12
  C2  32 rows, fp32 Student-t(nu=3) * 2.5
  C3  256 rows, bf16 N(0, 4^2) - 1.1 * ln(rank), rank = seeded permutation + 1
  C4  64 hidden rows of width 2560 (N(0,1), RMS-normalised) and a
      262144 x 2560 Q4_0 LM head (reference interleaved layout)
  C5  1024 rows, fp32 N(0, 3^2), per-row T ~ U[0.3,1.5], K in {1,20,64,200},
      P ~ U[0.5, 1]
"""
from __future__ import annotations

import numpy as np

V = 262144
SEEDS = {"c1": 0xC1, "c2": 0xC2, "c3": 0xC3, "c4": 0xC4, "c5": 0xC5}


def rng(seed: int, step: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(np.random.SeedSequence([seed, step])))


def f32_to_bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def uniforms(n: int, seed: int, step: int = 0) -> np.ndarray:
    return rng(seed ^ 0x5EED, step).random(n)


def c1_logits(step: int, vocab: int = V, seed: int = SEEDS["c1"]) -> np.ndarray:
    g = rng(seed, step)
    x = (g.standard_normal(vocab) * 3.0).astype(np.float32)
    spikes = g.choice(vocab, size=min(16, vocab), replace=False)
    x[spikes] += np.float32(12.0)
    return x


def c2_logits(rows: int = 32, vocab: int = V, seed: int = SEEDS["c2"], step: int = 0) -> np.ndarray:
    g = rng(seed, step)
    z = g.standard_normal((rows, vocab))
    chi2 = g.chisquare(3, size=(rows, vocab))
    return (z / np.sqrt(chi2 / 3.0) * 2.5).astype(np.float32)


def c3_logits(rows: int = 256, vocab: int = V, seed: int = SEEDS["c3"], step: int = 0) -> np.ndarray:
    """bf16 bit patterns (uint16) [rows, vocab]."""
    g = rng(seed, step)
    out = np.empty((rows, vocab), dtype=np.uint16)
    lnr = np.log(np.arange(1, vocab + 1, dtype=np.float64))
    for r in range(rows):
        perm = g.permutation(vocab)
        x = g.standard_normal(vocab) * 4.0 - 1.1 * lnr[perm]
        out[r] = f32_to_bf16_rne(x.astype(np.float32))
    return out


def c5_logits(rows: int = 1024, vocab: int = V, seed: int = SEEDS["c5"], step: int = 0) -> np.ndarray:
    g = rng(seed, step)
    return (g.standard_normal((rows, vocab)) * 3.0).astype(np.float32)


def c5_params(rows: int = 1024, seed: int = SEEDS["c5"]):
    """Per-row (temperature, top_k, top_p)."""
    g = rng(seed ^ 0xAA, 0)
    t = g.uniform(0.3, 1.5, rows).astype(np.float32)
    k = g.choice(np.array([1, 20, 64, 200]), size=rows)
    p = g.uniform(0.5, 1.0, rows).astype(np.float32)
    return [(float(t[i]), int(k[i]), float(p[i])) for i in range(rows)]


def f32_to_f16_rne(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def c4_inputs(rows: int = 64, hidden: int = 2560, vocab: int = V, seed: int = SEEDS["c4"]):
    """(hidden fp32 [rows, hidden], Q4_0 blocks uint8 [vocab * hidden/32 * 18]).

    Block layout (src/Gemma4.Types.pas:139-142): little-endian fp16 scale, then
    16 bytes; byte j holds element 2j in its low nibble and 2j+1 in its high
    nibble; element value = nibble - 8.
    """
    g = rng(seed, 0)
    h = g.standard_normal((rows, hidden)).astype(np.float32)
    h = (h / np.sqrt(np.mean(h.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)).astype(np.float32)
    nblk = vocab * (hidden // 32)
    q = g.integers(-8, 8, size=(nblk, 32), dtype=np.int16) + 8  # stored nibble = q + 8
    q = q.astype(np.uint8)
    scales = f32_to_f16_rne(g.uniform(0.002, 0.02, nblk).astype(np.float32))
    blocks = np.empty((nblk, 18), dtype=np.uint8)
    blocks[:, 0] = (scales & 0xFF).astype(np.uint8)
    blocks[:, 1] = (scales >> 8).astype(np.uint8)
    blocks[:, 2:] = q[:, 0::2] | (q[:, 1::2] << 4)
    return h, blocks.reshape(-1)
