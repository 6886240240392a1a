"""RoPE tables of the C ABI's host entry points against the oracle.

ncm_rope_tables_host and ncm_rope_tables_llama3_host are host functions of
libncm_cuda.so (no device needed): the tables the GPU attention reads, at the
per-level restarting positions of src/ncm_position.zig:11-22. They must equal
the oracle's restatement of rope_default / rope_llama3 + rope_tables
(packages/kernels/root.zig:305-348, :636-674) bit for bit.
"""
import numpy as np
import pytest

# Llama-3.2-1B's rope_scaling (packages/hf_config/testdata/llama-3.2-1b/config.json)
LLAMA32 = (32.0, 1.0, 4.0, 8192)


def _positions():
    from ncmorph_b200.ncm_model import level_positions
    return level_positions(1, [256, 256, 512, 1024, 2048])


@pytest.mark.parametrize("theta", [500000.0, 10000.0])
def test_default_tables_match_oracle(orc, theta):
    from ncmorph_b200.ncm_model import rope_tables
    pos = _positions()
    c, s = rope_tables(64, theta, pos)
    _, oc, os_ = orc.rope_default(64, theta, int(pos.max()) + 1)
    assert np.array_equal(c.view(np.uint32), oc[pos].view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_[pos].view(np.uint32))


@pytest.mark.parametrize("head_dim,theta,scaling", [(64, 500000.0, LLAMA32), (128, 500000.0, (8.0, 1.0, 4.0, 8192)),
                                                    (64, 10000.0, (4.0, 2.0, 8.0, 2048))])
def test_llama3_tables_match_oracle(orc, head_dim, theta, scaling):
    from ncmorph_b200.ncm_model import rope_tables
    pos = _positions()
    c, s = rope_tables(head_dim, theta, pos, llama3=scaling)
    inv = orc.rope_llama3(head_dim, theta, *scaling)
    oc, os_ = orc.rope_tables(inv, int(pos.max()) + 1)
    assert np.array_equal(c.view(np.uint32), oc[pos].view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_[pos].view(np.uint32))
    # the scaling changes the low frequencies (otherwise this test would not see it)
    _, dc, _ = orc.rope_default(head_dim, theta, int(pos.max()) + 1)
    assert not np.array_equal(oc, dc)


def test_llama3_rejects_what_the_reference_asserts():
    from ncmorph_b200 import _lib
    from ncmorph_b200.ncm_model import rope_tables
    pos = _positions()
    for bad in [(0.0, 1.0, 4.0, 8192), (32.0, 0.0, 4.0, 8192), (32.0, 4.0, 4.0, 8192), (32.0, 1.0, 4.0, 0)]:
        with pytest.raises(_lib.NcmError) as e:
            rope_tables(64, 500000.0, pos, llama3=bad)
        assert e.value.status == _lib.NCM_EINVAL
    with pytest.raises(_lib.NcmError):
        rope_tables(63, 500000.0, pos, llama3=LLAMA32)
