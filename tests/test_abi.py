"""CPU tests of the C ABI library: it loads, exports every entry point that
include/pokit_cuda.h declares, and rejects invalid arguments before touching
a device (no compute call runs here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from pokitlms_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def so():
    build.build()
    return _lib.lib()


def declared_symbols():
    text = (ROOT / "include" / "pokit_cuda.h").read_text()
    return sorted(set(re.findall(r"\b(pokit_cuda_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    syms = declared_symbols()
    for s in ("pokit_cuda_linear", "pokit_cuda_moe_forward", "pokit_cuda_moe_create",
              "pokit_cuda_linear_backend_try_linear", "pokit_cuda_moe_expert_view"):
        assert s in syms


def test_every_declared_symbol_is_exported(so):
    missing = [s for s in declared_symbols() if not hasattr(so, s)]
    assert not missing, missing
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "binding and header disagree"


def test_library_has_no_torch_dependency():
    import subprocess
    out = subprocess.run(["ldd", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    assert "torch" not in out and "libcudart.so" not in out


def test_version(so):
    assert so.pokit_cuda_version().decode() == "0.1.0"


def test_invalid_moe_config_is_rejected(so):
    cfg = _lib.MoeConfig(0, 1, 2000, 768, 128, 8, 0, 1, 1.0, 1e-6, 12, 12, 12, None, 0, 8, 8, 8)
    h = C.c_void_p()
    err = _lib.ErrorBuffer()
    st = so.pokit_cuda_moe_create(C.byref(cfg), C.byref(h), *err.args())
    assert st == _lib.STATUS_INVALID_ARGUMENT and not h.value
    assert "invalid MoE configuration" in err.text()
    cfg = _lib.MoeConfig(0, 1, 2048, 768, 128, 200, 0, 1, 1.0, 1e-6, 12, 12, 12, None, 0, 8, 8, 8)
    assert so.pokit_cuda_moe_create(C.byref(cfg), C.byref(h), *err.args()) == 1
    cfg = _lib.MoeConfig(0, 1, 2048, 768, 128, 8, 0, 1, 1.0, 1e-6, 2, 12, 12, None, 0, 8, 8, 8)
    assert so.pokit_cuda_moe_create(C.byref(cfg), C.byref(h), *err.args()) == 1
    assert so.pokit_cuda_moe_create(None, C.byref(h), *err.args()) == 1


def test_invalid_linear_arguments_are_rejected(so):
    err = _lib.ErrorBuffer()
    assert so.pokit_cuda_linear(2, 1, 4, 32, 1, 1, None, *err.args()) == 1      # Q4_0 unsupported
    assert so.pokit_cuda_linear(12, 1, 4, 100, 1, 1, None, *err.args()) == 1    # cols % 256
    assert so.pokit_cuda_linear(12, None, 4, 256, 1, 1, None, *err.args()) == 1
    assert so.pokit_cuda_route_experts(1, 4, 5, 0, 1, 1.0, 1, 1, None, None, *err.args()) == 1
    assert so.pokit_cuda_route_experts(1, 4, 2, 3, 1, 1.0, 1, 1, None, None, *err.args()) == 1
    assert so.pokit_cuda_synthesize_blocks(0, 0, 0, 1, 1, None, *err.args()) == 1


def test_error_buffer_truncation(so):
    buf = C.create_string_buffer(8)
    assert so.pokit_cuda_linear(2, 1, 4, 32, 1, 1, None, buf, 8) == 1
    assert len(buf.value) == 7
    assert so.pokit_cuda_linear(2, 1, 4, 32, 1, 1, None, None, 0) == 1


def test_null_handles(so):
    assert so.pokit_cuda_moe_get_stats(None, None) == 1
    assert so.pokit_cuda_linear_backend_get_stats(None, None) == 1
    assert so.pokit_cuda_moe_tensor_bytes(None, 0, 0) == 0
    so.pokit_cuda_moe_destroy(None)
    so.pokit_cuda_linear_backend_destroy(None)
