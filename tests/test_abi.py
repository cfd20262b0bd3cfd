"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls: these run without a GPU)."""

import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from g2ptq_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from g2ptq_b200.build import build
        build()
    return _lib.load()


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*[\w\s\*]+?\b(g2q_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "g2q_gram_update" in names and "g2q_compensate" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_binding_covers_every_declared_symbol():
    from g2ptq_b200 import _lib
    missing = [n for n in declared_functions() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_abi_version_and_status_strings(lib):
    from g2ptq_b200 import _lib
    assert lib.g2q_abi_version() == _lib.ABI_VERSION
    assert _lib.status_string(_lib.G2Q_ERR_BAD_SCALE) == "non-positive quantization scale"
    assert _lib.status_string(7) == "non-positive Cholesky pivot"


def test_invalid_arguments_rejected_without_gpu(lib):
    # argument validation happens on the host before any CUDA call
    assert lib.g2q_gemm(None, 0, 0, None, 0, 0, 0, None, 0, 0, 0, 1, 1, 1, 1,
                        ctypes.c_float(0), ctypes.c_float(1), 0, None) == -1
    assert lib.g2q_compensate_block(0, None, 0, 0, 0, 0, 0, None, 0, 0, None, None, 0, None,
                                    7, None, None, None, None, None, None, 0.0, None) == -1
    assert lib.g2q_pack_int32(None, None, 1, 1, 4, None) == -1


def test_ops_refuse_cpu_tensors():
    import torch
    from g2ptq_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.argsort_desc(torch.zeros(4))


def test_workspace_queries(lib):
    from g2ptq_b200 import _lib
    assert _lib.query("g2q_chol_workspace_bytes", 4096) >= 2 * 4096 * 4096 * 4
    assert _lib.query("g2q_compensate_workspace_bytes", 0, 1, 4096, 4096, 0) >= 4096 * 128 * 4


def test_wait_limit_is_settable_on_the_host(lib):
    # host-side setting read by every tensor-core launch; no GPU call here
    default = 4_000_000_000
    prev = lib.g2q_set_wait_limit(1000)
    try:
        assert prev == default
        assert lib.g2q_set_wait_limit(0) == 1000  # 0 restores the default
        assert lib.g2q_set_wait_limit(-5) == default
    finally:
        lib.g2q_set_wait_limit(0)
    assert lib.g2q_set_wait_limit(0) == default
