"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/epb.h declares, and rejects bad configurations before touching CUDA."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "epb.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(epb_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from dreamplacett_framework_b200 import _lib, build
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    from dreamplacett_framework_b200 import _lib
    names = _declared()
    assert len(names) >= 13
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTS)


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.epb_version()
    assert lib.epb_status_string(0) == b"ok"
    assert lib.epb_status_string(5) == b"fixed-point density saturated"


def test_create_rejects_bad_config_without_cuda(lib):
    from dreamplacett_framework_b200 import _lib
    h = ctypes.c_void_p()
    assert lib.epb_create(None, ctypes.byref(h)) == _lib.EPB_EINVAL
    for M, N, box in ((100, 64, (0, 0, 1, 1)), (64, 8, (0, 0, 1, 1)), (8192, 64, (0, 0, 1, 1)),
                      (64, 64, (0, 0, 0, 1)), (64, 64, (0, 0, float("nan"), 1))):
        cfg = _lib.EpbConfig(M, N, *box, 0, 0, 0, 0)
        assert lib.epb_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.EPB_EINVAL
        assert not h.value
    cfg = _lib.EpbConfig(64, 64, 0, 0, 1, 1, 0, 0, 7, 0)  # flags must be 0
    assert lib.epb_create(ctypes.byref(cfg), ctypes.byref(h)) == _lib.EPB_EINVAL


def test_null_handle_calls_fail_cleanly(lib):
    from dreamplacett_framework_b200 import _lib
    assert lib.epb_destroy(None) == _lib.EPB_EINVAL
    assert lib.epb_forward(None, None, None, None, None, None, None, None) == _lib.EPB_EINVAL
    assert lib.epb_backward(None, None, None, None, None, None) == _lib.EPB_EINVAL
    assert lib.epb_last_error(None) == b"null handle"


def test_struct_layout_matches_header():
    from dreamplacett_framework_b200 import _lib
    # epb_config: 2 x int32, 4 x double, 4 x int32 -> 56 bytes; epb_cells: 7 pointers + 4 x int64
    assert ctypes.sizeof(_lib.EpbConfig) == 56
    assert ctypes.sizeof(_lib.EpbCells) == 7 * 8 + 4 * 8


def test_engine_refuses_cpu_only():
    import torch
    from dreamplacett_framework_b200.engine import ElectricPotentialEngine
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    with pytest.raises(RuntimeError, match="CUDA"):
        ElectricPotentialEngine(64, 64, 0, 0, 100, 100)
