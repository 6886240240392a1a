"""Generates the committed golden fixtures in tests/golden/ from the ncmorph
reference checkout (run in the build container, where the reference is
mounted; the GPU box never needs the reference).

  python tests/golden/gen_golden.py <path-to-ncmorph-checkout>

Outputs
  bf16_pairs.txt   the 4,119 (f32 bits, bf16 bits) pairs of
                   packages/bf16/vectors.zig (PyTorch-generated, read as data)
  pool_area.npz    torch F.interpolate(mode="area") outputs on seeded inputs,
                   pinning the pooling semantics R4 restates
"""
from __future__ import annotations

import pathlib
import re
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def bf16_pairs(ref_root: pathlib.Path) -> None:
    text = (ref_root / "packages" / "bf16" / "vectors.zig").read_text()
    pairs = re.findall(r"\.\{\s*0x([0-9A-Fa-f]{8}),\s*0x([0-9A-Fa-f]{4})\s*\}", text)
    if len(pairs) != 4119:
        raise SystemExit(f"expected 4119 pairs, found {len(pairs)}")
    with open(HERE / "bf16_pairs.txt", "w") as f:
        f.write("# f32_bits bf16_bits — from ncmorph packages/bf16/vectors.zig (PyTorch 2.13.0)\n")
        for a, b in pairs:
            f.write(f"{a.upper()} {b.upper()}\n")


def pool_area() -> None:
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(1234)
    out = {}
    for (B, T, D, f) in [(2, 64, 24, 16), (1, 48, 8, 4), (3, 32, 16, 2), (2, 16, 8, 1)]:
        x = torch.randn(B, T, D, generator=g, dtype=torch.float32)
        y = F.interpolate(x.transpose(1, 2), size=T // f, mode="area").transpose(1, 2).contiguous()
        out[f"x_{B}_{T}_{D}_{f}"] = x.numpy()
        out[f"y_{B}_{T}_{D}_{f}"] = y.numpy()
    np.savez_compressed(HERE / "pool_area.npz", **out)


if __name__ == "__main__":
    ref = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    bf16_pairs(ref)
    pool_area()
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".txt", ".npz")))
