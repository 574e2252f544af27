"""Generates the golden fixtures in this folder from the reference's own
flash_attention_forward (FlashAttention.cpp:24-182) and flash_attention_backward
(FlashAttention.cpp:185-359), compiled in place from the DirkTensor sources into
oracle/_ref (see oracle/Makefile).

Inputs are not stored: they are regenerated from the seeds with
numpy.random.default_rng (PCG64, standard_normal float32) and checked against a
stored checksum.  flash_ref.npz: o [B,T,H,D], m and l [B,T,H] (float32).
flash_bwd_ref.npz: dq, dk, dv [B,T,H,D] for an upstream gradient dO drawn from
seed + 1000, with o, m, l taken from the reference's own forward.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle  # noqa: E402
from common import SCALE, qkv, randn  # noqa: E402

# (name, seed, B, T, H, causal): edge lengths around the 128/256 tile sizes,
# a one-token sequence, a batch of 2, and one non-causal case.
CASES = [
    ("t1", 11, 1, 1, 2, True),
    ("t63", 12, 1, 63, 2, True),
    ("t65", 13, 1, 65, 2, True),
    ("t129_b2", 14, 2, 129, 1, True),
    ("t257", 15, 1, 257, 2, True),
    ("t300_full", 16, 1, 300, 1, False),
    ("t520_h1", 17, 1, 520, 1, True),
]

# backward cases: a single token, tile edges, a batch of 2, non-causal
BWD_CASES = [
    ("t1", 21, 1, 1, 2, True),
    ("t129_b2", 22, 2, 129, 1, True),
    ("t257", 23, 1, 257, 2, True),
    ("t300_full", 24, 1, 300, 1, False),
]


def checksum(*arrs) -> float:
    return float(sum(np.sum(a.astype(np.float64) * (1 + np.arange(a.size).reshape(a.shape) % 7)) for a in arrs))


def main() -> None:
    if oracle.ref_lib() is None:
        oracle.build(with_reference=True)
    out = {}
    for name, seed, B, T, H, causal in CASES:
        q, k, v = qkv(seed, B, T, H)
        o, m, l, _ = oracle.ref_flash_fwd(q, k, v, SCALE, causal)
        out[f"{name}__meta"] = np.array([seed, B, T, H, int(causal)], np.int64)
        out[f"{name}__checksum"] = np.array([checksum(q, k, v)], np.float64)
        out[f"{name}__o"] = o
        out[f"{name}__m"] = m
        out[f"{name}__l"] = l
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "flash_ref.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")
    out = {}
    for name, seed, B, T, H, causal in BWD_CASES:
        q, k, v = qkv(seed, B, T, H)
        do = randn(seed + 1000, q.shape)
        o, m, l, _ = oracle.ref_flash_fwd(q, k, v, SCALE, causal)
        dq, dk, dv, _ = oracle.ref_flash_bwd(do, o, m, l, q, k, v, SCALE, causal)
        out[f"{name}__meta"] = np.array([seed, B, T, H, int(causal)], np.int64)
        out[f"{name}__checksum"] = np.array([checksum(q, k, v, do)], np.float64)
        out[f"{name}__dq"] = dq
        out[f"{name}__dk"] = dk
        out[f"{name}__dv"] = dv
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "flash_bwd_ref.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
