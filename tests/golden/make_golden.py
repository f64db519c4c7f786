"""Generate the golden fixtures in tests/golden/ (committed; re-run to refresh).

The reference pins no numerics for the GEMM path (it zero-fills A and B and
never reads D: cutlass_gemm_mainloop/cutlass_gemm_bench.cu:71-75,180-185), so
these fixtures come from independent restatements, not from the C oracle:

  * rng.npz      -- splitmix64 bits computed with Python integers, the uniform
                    grid from those bits, and Box-Muller normals computed with
                    numpy's libm log/cos in float64 (the oracle uses its own
                    series for ln/cos and must agree to the last float32 bit
                    on these draws).
  * quant.npz    -- bf16 and e4m3 roundings from PyTorch's dtype casts
                    (torch.bfloat16, torch.float8_e4m3fn), on values inside the
                    e4m3 finite range.
  * nvfp4.npz    -- NVFP4 quantisation (absmax/6 scale rounded up to unsigned
                    e4m3, e2m1 round-to-nearest-even) restated in numpy over
                    the golden normals, with the interleaved scale layout.
  * gemm.npz     -- small GEMMs D = A . B^T in float64 with numpy over bf16-
                    and e4m3-representable inputs taken from torch casts.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
MASK = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


def mix64(z: int) -> int:
    z &= MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
    return z ^ (z >> 31)


def bits(seed: int, stream: int, idx: int) -> int:
    key = mix64(seed + mix64(stream + GOLDEN))
    return mix64(key + (idx + 1) * GOLDEN)


def uniform(b: int) -> float:
    return np.float32((b >> 40)) * np.float32(1.0 / 8388608.0) - np.float32(1.0)


def normal(b: int) -> np.float32:
    u1 = ((b >> 32) + 1.0) / 4294967296.0
    u2 = (b & 0xFFFFFFFF) / 4294967296.0
    return np.float32(np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2))


E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def e4m3_values() -> np.ndarray:
    """All non-negative finite e4m3 values indexed by code 0..126."""
    codes = torch.arange(0, 127, dtype=torch.uint8)
    return codes.view(torch.float8_e4m3fn).to(torch.float64).numpy()


def e2m1_rne(x: float) -> int:
    a = abs(x)
    if a >= 6.0:
        c = 7
    else:
        d = np.abs(E2M1 - a)
        best = np.flatnonzero(d == d.min())
        c = int(best[0]) if len(best) == 1 else int(best[best % 2 == 0][0])  # tie -> even code
    return (8 if np.signbit(np.float32(x)) else 0) | c


def nvfp4_block(v: np.ndarray, e4m3: np.ndarray):
    amax = np.float32(np.abs(v).max())
    t = np.float32(amax / np.float32(6.0))
    if not t > 0:
        return 0, np.zeros(16, dtype=np.uint8)
    idx = int(np.searchsorted(e4m3, float(t), side="left"))   # smallest code with value >= t
    idx = min(idx, 126)
    s = np.float32(e4m3[idx])
    q = np.array([e2m1_rne(float(np.float32(x / s))) for x in v], dtype=np.uint8)
    return idx, q


def sf_offset(r: int, c: int, cols: int) -> int:
    kblocks = cols // 64
    return ((r // 128) * kblocks + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (c % 4)


def main() -> None:
    # ---------------------------------------------------------------- rng
    idx = list(range(0, 4096)) + [10**6 + i for i in range(64)] + [2**40 + i for i in range(64)]
    cases = [(0, 0), (0, 1), (7, 3), (123456789, 42)]
    rows = []
    for seed, stream in cases:
        for i in idx:
            rows.append((seed, stream, i, bits(seed, stream, i)))
    arr = np.array(rows, dtype=np.uint64)
    u = np.array([uniform(int(b)) for b in arr[:, 3]], dtype=np.float32)
    nrm = np.array([normal(int(b)) for b in arr[:, 3]], dtype=np.float32)
    np.savez_compressed(OUT / "rng.npz", seed=arr[:, 0], stream=arr[:, 1], idx=arr[:, 2],
                        bits=arr[:, 3], uniform=u, normal=nrm)

    # ---------------------------------------------------------------- quant
    g = np.random.default_rng(2024)
    x = np.concatenate([g.standard_normal(5000).astype(np.float32) * s
                        for s in (1e-5, 1e-3, 0.02, 0.25, 1.0, 30.0, 200.0)])
    x = x[np.abs(x) < 440.0]
    ties = np.array([0.0, -0.0, 2 ** -10, 3 * 2 ** -10, 1.0 + 2 ** -4, 1.0 + 3 * 2 ** -4, 448.0, -448.0],
                    dtype=np.float32)
    x = np.concatenate([x, ties])
    t = torch.from_numpy(x)
    np.savez_compressed(OUT / "quant.npz", x=x,
                        bf16=t.to(torch.bfloat16).view(torch.uint16).numpy(),
                        e4m3=t.to(torch.float8_e4m3fn).view(torch.uint8).numpy())

    # ---------------------------------------------------------------- nvfp4
    e4m3 = e4m3_values()
    R, K = 128, 128
    vals = np.array([[normal(bits(0, 5, r * K + c)) for c in range(K)] for r in range(R)], dtype=np.float32)
    vals[3, 16:32] = 0.0                    # an all-zero block gets scale 0
    vals[5, 0:16] = np.float32(1e-6)        # a block below the smallest scale
    packed = np.zeros((R, K // 2), dtype=np.uint8)
    scales = np.zeros(((R + 127) // 128) * (K // 64) * 512, dtype=np.uint8)
    for r in range(R):
        for cb in range(K // 16):
            sq, q = nvfp4_block(vals[r, cb * 16:(cb + 1) * 16], e4m3)
            scales[sf_offset(r, cb, K)] = sq
            for j in range(0, 16, 2):
                packed[r, (cb * 16 + j) // 2] = q[j] | (q[j + 1] << 4)
    np.savez_compressed(OUT / "nvfp4.npz", values=vals, packed=packed, scales=scales)

    # ---------------------------------------------------------------- gemm
    out = {}
    for name, (m, n, k, dt) in {"bf16_64x48x96": (64, 48, 96, "bf16"),
                                "e4m3_32x40x128": (32, 40, 128, "e4m3"),
                                "bf16_1x1x1000": (1, 1, 1000, "bf16")}.items():
        a = torch.from_numpy(g.uniform(-1, 1, (m, k)).astype(np.float32))
        b = torch.from_numpy(g.uniform(-1, 1, (n, k)).astype(np.float32))
        if dt == "bf16":
            a, b = a.to(torch.bfloat16).float(), b.to(torch.bfloat16).float()
        else:
            a, b = a.to(torch.float8_e4m3fn).float(), b.to(torch.float8_e4m3fn).float()
        A, B = a.numpy(), b.numpy()
        out[name + "_A"] = A
        out[name + "_B"] = B
        out[name + "_D"] = A.astype(np.float64) @ B.astype(np.float64).T
    np.savez_compressed(OUT / "gemm.npz", **out)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
