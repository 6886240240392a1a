"""Device-side safetensors loading (ncm_load_tensor_bf16): BF16 tensors
arrive bit for bit; F16 and F32 arrive rounded to bf16 with the bf16
package's rule (checked against the oracle's restatement of
packages/bf16/root.zig:17-31). Sizes span several 16 MiB staging chunks (each read
by four threads)."""
import time

import numpy as np
import pytest
import torch

from helpers import from_dev_bf16
from test_loader_header import write_safetensors

pytestmark = pytest.mark.gpu


def test_load_bf16_f16_f32(orc, cuda_dev, tmp_path):
    from ncmorph_b200 import loader
    rng = np.random.default_rng(3)
    n_big = 3 * (16 << 20) // 2 + 12345           # bf16 tensor spanning 4 chunks, ragged tail
    bf = rng.integers(0, 1 << 16, size=n_big, dtype=np.uint16)
    f16 = rng.standard_normal(1 << 20).astype(np.float16)
    f16[:4] = [np.inf, -np.inf, 0.0, -0.0]
    f32 = (rng.standard_normal((1000, 4099)) * 3).astype(np.float32)
    f32.flat[:3] = [np.nan, 1.0039062, 3.3895314e38]   # NaN, a tie, rounds to inf
    p = tmp_path / "w.safetensors"
    write_safetensors(p, {"w_bf16": bf.tobytes(), "w_f16": f16.tobytes(), "w_f32": f32.tobytes()},
                      {"w_bf16": ("BF16", (n_big,)), "w_f16": ("F16", (1 << 20,)), "w_f32": ("F32", f32.shape)})
    got = loader.load_all_bf16(p, cuda_dev)
    t0 = time.time()
    loader.load_all_bf16(p, cuda_dev)        # second pass: staging allocated, file in the page cache
    torch.cuda.synchronize()
    dt = time.time() - t0
    total = bf.nbytes + f16.nbytes + f32.nbytes
    print(f"loaded {total / 1e6:.1f} MB in {dt * 1e3:.1f} ms ({total / dt / 1e9:.2f} GB/s, page cache)")
    assert np.array_equal(from_dev_bf16(got["w_bf16"]), bf)
    assert np.array_equal(from_dev_bf16(got["w_f16"]), orc.bf16_bits(f16.astype(np.float32)))
    assert np.array_equal(from_dev_bf16(got["w_f32"]).reshape(f32.shape), orc.bf16_bits(f32))


def test_load_rejects_bad_arguments(cuda_dev, tmp_path):
    from ncmorph_b200 import _lib, device
    lib = _lib.load()
    ctx = device.context(cuda_dev)
    out = torch.empty(4, dtype=torch.bfloat16, device=cuda_dev)
    rc = lib.ncm_load_tensor_bf16(ctx, str(tmp_path / "missing").encode(), 0, 8, 0, out.data_ptr(), None)
    assert rc == _lib.NCM_EINVAL
    rc = lib.ncm_load_tensor_bf16(ctx, b"/dev/null", 0, 6, 2, out.data_ptr(), None)   # 6 bytes of F32
    assert rc == _lib.NCM_EINVAL
