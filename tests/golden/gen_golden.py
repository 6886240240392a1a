"""Generates the committed golden fixtures in tests/golden/ from the ncmorph
reference checkout (run in the build container, where the reference is
mounted; the GPU box never needs the reference).

  python tests/golden/gen_golden.py <path-to-ncmorph-checkout>

Outputs
  bf16_pairs.txt   the 4,119 (f32 bits, bf16 bits) pairs of
                   packages/bf16/vectors.zig (PyTorch-generated, read as data)
  pool_area.npz    torch F.interpolate(mode="area") outputs on seeded inputs,
                   pinning the pooling semantics R4 restates
  upsample.npz     torch F.interpolate(mode="linear"/"nearest", size=T) outputs
                   (the quantiser's U_i, vq_forward_semantics.md:82)
  conv1d_k3.npz    torch F.conv1d(kernel 3, padding 1) in float64 on seeded
                   inputs (the Phi / post-upsample convolution)
  level0.npz       torch F.group_norm (affine=False), F.conv1d(kernel 4,
                   stride 4) and F.conv_transpose1d(kernel 4, stride 4) in
                   float64 (pre-quant GroupNorm and the level-0 cascade stage)
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


def upsample() -> None:
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(4321)
    out = {}
    for (B, Tq, D, T) in [(2, 16, 24, 256), (1, 37, 8, 100), (3, 16, 16, 32), (2, 5, 8, 5), (1, 1, 8, 16)]:
        q = torch.randn(B, Tq, D, generator=g, dtype=torch.float32)
        out[f"q_{B}_{Tq}_{D}_{T}"] = q.numpy()
        for mode in ("linear", "nearest"):
            y = F.interpolate(q.transpose(1, 2), size=T, mode=mode).transpose(1, 2).contiguous()
            out[f"{mode}_{B}_{Tq}_{D}_{T}"] = y.numpy()
    np.savez_compressed(HERE / "upsample.npz", **out)


def conv1d_k3() -> None:
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(99)
    out = {}
    for (T, C) in [(50, 24), (7, 3), (1, 8), (33, 64)]:
        x = torch.randn(T, C, generator=g, dtype=torch.float32)
        w = torch.randn(C, C, 3, generator=g, dtype=torch.float32) * 0.1
        b = torch.randn(C, generator=g, dtype=torch.float32)
        y = F.conv1d(x.T[None].double(), w.double(), b.double(), padding=1)[0].T.contiguous()
        out[f"x_{T}_{C}"], out[f"w_{T}_{C}"], out[f"b_{T}_{C}"] = x.numpy(), w.numpy(), b.numpy()
        out[f"y_{T}_{C}"] = y.numpy()
    np.savez_compressed(HERE / "conv1d_k3.npz", **out)


def level0() -> None:
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(777)
    out = {}
    x = torch.randn(2, 32, 24, generator=g, dtype=torch.float32)
    out["gn_x"] = x.numpy()
    out["gn_y"] = F.group_norm(x.transpose(1, 2).double(), 8, eps=1e-5).transpose(1, 2).contiguous().numpy()
    w = torch.randn(24, 24, 4, generator=g, dtype=torch.float32) * 0.1
    b = torch.randn(24, generator=g, dtype=torch.float32)
    out["conv_x"], out["conv_w"], out["conv_b"] = x.numpy(), w.numpy(), b.numpy()
    xt = x.transpose(1, 2).double()
    out["down_y"] = F.conv1d(xt, w.double(), b.double(), stride=4).transpose(1, 2).contiguous().numpy()
    out["up_y"] = F.conv_transpose1d(xt, w.double(), b.double(), stride=4).transpose(1, 2).contiguous().numpy()
    np.savez_compressed(HERE / "level0.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_golden.py <path-to-ncmorph-checkout>")
    bf16_pairs(pathlib.Path(sys.argv[1]))
    pool_area()
    upsample()
    conv1d_k3()
    level0()
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".txt", ".npz")))
