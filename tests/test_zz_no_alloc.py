"""The no-allocation RVQ level entry point, through the C ABI.

Some callers cannot call cudaMalloc: host plugins whose application owns every
device allocation (its own arena or caching allocator must account for all
memory), and latency-bound paths that may not stall on cudaMalloc, which can
synchronise the device. ncm_rvq_level_noalloc serves them: it takes no context
and keeps its scratch in a fixed device array inside the library. Device-side
failures accumulate in that array's error word, which
ncm_rvq_level_noalloc_status reads and clears.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test. It must pass alone in a fresh
process and after the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


def _noalloc(residual, codebook, sqnorm, codes):
    from ncmorph_b200 import _lib
    N, D = residual.shape
    K = codebook.shape[0]
    vp = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream(residual.device).cuda_stream)
    return _lib.load().ncm_rvq_level_noalloc(vp(residual), vp(codebook), vp(sqnorm), vp(codes), N, D, K, stream)


def _status(dev):
    from ncmorph_b200 import _lib
    flags = ctypes.c_int32(-1)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    rc = _lib.load().ncm_rvq_level_noalloc_status(stream, ctypes.byref(flags))
    return rc, flags.value


def _case(dev, N, D, K, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    r = torch.randn((N, D), generator=g, device=dev)
    cb = torch.randn((K, D), generator=g, device=dev).to(torch.bfloat16)
    return r, cb


def _compare(dev, N, D, K, seed, give_norms):
    from ncmorph_b200 import vq
    r, cb = _case(dev, N, D, K, seed)
    sq = vq.code_sqnorm(cb)
    r_ref = r.clone()
    codes_ref = vq.rvq_level(r_ref, cb, sq)
    r_na = r.clone()
    codes_na = torch.full((N,), -1, dtype=torch.int32, device=dev)
    rc = _noalloc(r_na, cb, sq if give_norms else None, codes_na)
    assert rc == 0
    torch.cuda.synchronize()
    # same plan, kernels and arithmetic: codes and the f32 residual update match exactly
    assert torch.equal(codes_na, codes_ref), f"codes differ (N={N} D={D} K={K})"
    assert torch.equal(r_na, r_ref), f"residual differs (N={N} D={D} K={K})"


def test_noalloc_first_call_holds_at_most_its_array(cuda_dev):
    # The first call in a fresh process loads the module that holds the fixed
    # scratch array; free device memory may drop by that array (plus module
    # code), never by a workspace sized to the problem.
    r, cb = _case(cuda_dev, 2048, 512, 2048, 3)
    codes = torch.empty((2048,), dtype=torch.int32, device=cuda_dev)
    r1 = r.clone()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_dev)
    assert _noalloc(r1, cb, None, codes) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_dev)
    assert free0 - free1 <= SCRATCH_BYTES + (16 << 20)


def test_noalloc_matches_rvq_level_on_two_calls(cuda_dev):
    # First call: config-1 level shape with caller-supplied norms (code-split
    # partials in the scratch). Second call: smaller and
    # ragged, norms computed in the scratch; the first call's leftovers must
    # not leak into it.
    _compare(cuda_dev, 4096, 256, 1024, 1, True)
    _compare(cuda_dev, 1000, 136, 700, 2, False)
    assert _status(cuda_dev) == (0, 0)


def test_noalloc_matches_rvq_level_on_the_cta_pair_plan(cuda_dev):
    # 20480 rows: enough 256-row units for every CTA pair, so both entry points
    # run the pair kernel with the update fused (about 10 MiB of scratch)
    _compare(cuda_dev, 20480, 256, 1024, 4, True)


def test_noalloc_drops_split_partials_that_do_not_fit(cuda_dev):
    # 8192 x 1016 bf16 rows fill the scratch, so the two-split plan's partials
    # no longer fit and the call runs one split per row block; the result is
    # the same argmin and update as ncm_rvq_level's split plan
    _compare(cuda_dev, 8192, 1016, 4096, 5, False)


def test_noalloc_allocates_nothing_after_setup(cuda_dev):
    r, cb = _case(cuda_dev, 2048, 512, 2048, 3)
    codes = torch.empty((2048,), dtype=torch.int32, device=cuda_dev)
    assert _noalloc(r.clone(), cb, None, codes) == 0          # set-up call in this context
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_dev)
    for _ in range(3):
        assert _noalloc(r, cb, None, codes) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_dev)
    assert free1 == free0


def test_noalloc_status_reads_and_clears(cuda_dev):
    r, cb = _case(cuda_dev, 4096, 256, 1024, 6)
    codes = torch.empty((4096,), dtype=torch.int32, device=cuda_dev)
    for _ in range(2):
        assert _noalloc(r, cb, None, codes) == 0
        assert _status(cuda_dev) == (0, 0)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_dev):
    from ncmorph_b200 import _lib
    # 4096 x 4096 bf16 rows need 32 MiB of scratch, beyond the fixed 16 MiB
    r = torch.zeros((4096, 4096), device=cuda_dev)
    cb = torch.zeros((8, 4096), dtype=torch.bfloat16, device=cuda_dev)
    codes = torch.empty((4096,), dtype=torch.int32, device=cuda_dev)
    assert _noalloc(r, cb, None, codes) == _lib.NCM_EINVAL
    assert b"scratch" in _lib.load().ncm_last_error()
