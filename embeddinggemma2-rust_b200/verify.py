"""Parity tolerance profiles and checks, restating src/verify.rs:15-219.

A run's outputs pass when, per checked vector, max |got - want| stays within the profile's bound
and, where the profile has one, the cosine similarity (computed in f64) reaches its floor. NaN
fails, as does a length mismatch.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

TOL_EMBEDDING = 5e-6
TOL_SOFT_TOKENS = 1e-3
TOL_PIXELS = 1e-6
TOL_MEL = 1e-5


@dataclass(frozen=True)
class Limit:
    kind: str
    max_abs: float
    min_cos: float | None = None


@dataclass(frozen=True)
class Tolerances:
    name: str
    embedding: Limit
    soft_tokens: Limit
    pixels: Limit
    mel: Limit


FLOAT32 = Tolerances(
    "float32",
    Limit("embeddings", TOL_EMBEDDING),
    Limit("soft tokens", TOL_SOFT_TOKENS),
    Limit("patches", TOL_PIXELS),
    Limit("log-mel", TOL_MEL),
)
TF32 = Tolerances(
    "tf32",
    Limit("embeddings", 1e-3, 0.99999),
    Limit("soft tokens", 5e-1, 0.99999),
    FLOAT32.pixels,
    FLOAT32.mel,
)
BF16 = Tolerances(
    "bf16",
    Limit("embeddings", 4e-3, 0.99991),
    Limit("soft tokens", 3.5, 0.9996),
    FLOAT32.pixels,
    FLOAT32.mel,
)
PROFILES = {"f32": FLOAT32, "fp32": FLOAT32, "float32": FLOAT32, "tf32": TF32, "bf16": BF16}


def for_precision(precision: str | int) -> Tolerances:
    """The profile of a device precision (src/verify.rs:112-118): 0/f32, 1/tf32, 2/bf16."""
    if isinstance(precision, int):
        return (FLOAT32, TF32, BF16)[precision]
    return PROFILES[precision]


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(np.dot(a, b) / (np.sqrt(np.dot(a, a)) * np.sqrt(np.dot(b, b))))


def max_abs_diff(a, b) -> float:
    a = np.asarray(a, dtype=np.float32).ravel()
    b = np.asarray(b, dtype=np.float32).ravel()
    if a.shape != b.shape:
        return math.inf
    if a.size == 0:
        return 0.0
    d = np.abs(a.astype(np.float64) - b.astype(np.float64))
    if np.isnan(d).any():
        return math.nan
    return float(d.max())


@dataclass
class Check:
    label: str
    max_abs: float
    cos: float | None
    limit: Limit
    ids_ok: bool | None = None

    def passed(self) -> bool:
        """src/verify.rs:151-157 (``>=`` on the cosine so that NaN fails)."""
        if not math.isfinite(self.max_abs) or not self.max_abs <= self.limit.max_abs:
            return False
        if self.limit.min_cos is not None and not (self.cos is not None and self.cos >= self.limit.min_cos):
            return False
        return self.ids_ok is None or self.ids_ok

    def __str__(self) -> str:
        s = f"{'PASS' if self.passed() else 'FAIL'} {self.label:<34} max|d|={self.max_abs:.2e}"
        if self.cos is not None:
            s += f"  cos={self.cos:.8f}"
        if not self.passed():
            s += f"  [limit max|d|<={self.limit.max_abs:.1e}"
            if self.limit.min_cos is not None:
                s += f", cos>={self.limit.min_cos}"
            s += "]"
        return s


def vec_check(label: str, got, want, limit: Limit, ids_ok: bool | None = None) -> Check:
    """One vector against its reference (src/verify.rs:221-240)."""
    got = np.asarray(got, dtype=np.float32).ravel()
    want = np.asarray(want, dtype=np.float32).ravel()
    mad = max_abs_diff(got, want)
    cos = cosine(got, want) if got.shape == want.shape and got.size else None
    if cos is not None and math.isnan(cos):
        cos = None
    return Check(label, mad, cos, limit, ids_ok)
