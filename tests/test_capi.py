"""C-ABI checks that need no GPU: libncm_cuda.so loads, exports every entry
point include/ncm_cuda.h declares, and fails cleanly (a status, no abort)
where no usable device exists."""
import ctypes
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "ncm_cuda.h"
LIB = ROOT / "ncmorph_b200" / "libncm_cuda.so"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"NCM_API\s+(?:const\s+)?\w+\s*\*?\s*(ncm_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("ncm_ctx_create", "ncm_linear_bf16", "ncm_rvq_level", "ncm_rvq_encode", "ncm_rvq_decode",
                 "ncm_pool_avg", "ncm_tokenizer_forward", "ncm_linear_bf16_host_f32"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    assert LIB.exists(), "build libncm_cuda.so first (python -m ncmorph_b200.build)"
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(ncm_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"not exported: {missing}"
    # nothing beyond the declared C ABI leaks out under the ncm_ prefix
    extra = sorted(exported - set(declared_symbols()))
    assert not extra, f"undeclared exports: {extra}"


def test_python_binding_covers_header():
    from ncmorph_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_library_loads_and_reports_status_strings():
    from ncmorph_b200 import _lib
    lib = _lib.load()
    assert lib.ncm_version() >= 100
    assert lib.ncm_status_string(_lib.NCM_EINVAL) == b"invalid argument"
    assert lib.ncm_status_string(_lib.NCM_ETIMEOUT) == b"device wait timed out"


def test_invalid_calls_return_status_without_device():
    from ncmorph_b200 import _lib
    lib = _lib.load()
    # a null context is rejected before any CUDA call
    rc = lib.ncm_linear_bf16(None, None, None, None, None, 1, 8, 1, None)
    assert rc == _lib.NCM_EINVAL
    assert b"null context" in lib.ncm_last_error()
    rc = lib.ncm_ctx_create(0, None)
    assert rc == _lib.NCM_EINVAL


def test_ctx_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from ncmorph_b200 import _lib
    lib = _lib.load()
    ctx = ctypes.c_void_p()
    rc = lib.ncm_ctx_create(0, ctypes.byref(ctx))
    assert rc in (_lib.NCM_ECUDA, _lib.NCM_EINVAL)
    assert ctx.value is None
    assert lib.ncm_last_error()


def test_comm_unique_id_without_gpu():
    """NCCL is loaded on demand; a unique id needs no GPU."""
    from ncmorph_b200 import _lib, sharded
    try:
        uid = sharded.comm_unique_id()
    except _lib.NcmError as e:
        assert e.status == _lib.NCM_ENOTSUP  # no libnccl on this host
        return
    assert len(uid) == 128 and any(uid)


def test_sharded_encode_without_communicator_is_rejected():
    from ncmorph_b200 import _lib
    lib = _lib.load()
    assert lib.ncm_rvq_encode_sharded(None, None, None, None, 1, None, None, 1, 8, 1, None) == _lib.NCM_EINVAL


def test_every_context_entry_point_rejects_a_null_context():
    """Each entry point whose first parameter is the context validates it
    before anything else: a null context returns NCM_EINVAL (no crash, no
    CUDA call). Run in a child process so a crash cannot take pytest down."""
    import re
    import subprocess
    import sys
    header = (ROOT / "include" / "ncm_cuda.h").read_text()
    # ncm_ctx_destroy(NULL) is a no-op that succeeds, as free(NULL) does
    names = [n for n in re.findall(r"NCM_API int (ncm_\w+)\(ncm_ctx_t\* ctx\b", header) if n != "ncm_ctx_destroy"]
    assert len(names) >= 30
    code = r'''
import ctypes, sys
from ncmorph_b200 import _lib
lib = _lib.load()
bad = []
for name in sys.argv[1:]:
    fn = getattr(lib, name)
    args = []
    for t in fn.argtypes:
        if t in (ctypes.c_int32, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32):
            args.append(1)
        elif t in (ctypes.c_float, ctypes.c_double):
            args.append(1.0)
        else:
            args.append(None)
    rc = fn(*args)
    if rc != _lib.NCM_EINVAL or b"null context" not in (lib.ncm_last_error() or b""):
        bad.append((name, rc))
print(bad)
'''
    out = subprocess.run([sys.executable, "-c", code, *names], capture_output=True, text=True, cwd=ROOT, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == "[]", out.stdout
