"""CPU tests of the C-ABI boundary: the library builds/loads, exports every
function include/agpu.h declares, the ctypes table covers the header, and the
calls that need no GPU behave (status strings, NULL handling, no device)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT, cuda_available

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions() -> list[str]:
    names = []
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"AGPU_API\s+[\w\s\*]+?\b(agpu_\w+)\s*\(", text)
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 30
    assert len(set(names)) == len(names)


def test_library_exports_every_declared_symbol():
    from any_gpu import _lib
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (agpu_\w+)", out))
    assert set(declared_functions()) <= exported


def _header_arities() -> dict:
    out = {}
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for name, params in re.findall(r"AGPU_API\s+[\w\s\*]+?\b(agpu_\w+)\s*\(([^;]*?)\)\s*;",
                                       text, flags=re.S):
            params = " ".join(params.split())
            out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_rust_ffi_matches_header():
    """The Rust crate's raw bindings (any-gpu_b200/rust/src/ffi.rs) declare
    every function of the header with the same number of arguments (it is not
    compiled in this image, so this keeps it in step with the header)."""
    ffi = (ROOT / "any-gpu_b200" / "rust" / "src" / "ffi.rs").read_text()
    rust = {}
    for name, params in re.findall(r"pub fn (agpu_\w+)\s*\(([^)]*)\)", ffi, flags=re.S):
        params = [p for p in params.split(",") if p.strip()]
        rust[name] = len(params)
    assert rust == _header_arities()
    device = (ROOT / "any-gpu_b200" / "rust" / "src" / "device.rs").read_text()
    for fn in ("pub fn gpu(", "pub fn upload(", "pub fn alloc(", "pub fn read(", "pub fn matmul(",
               "pub fn batch_matmul(", "pub fn softmax(", "pub fn scaled_dot_product_attention(",
               "pub fn conv2d(", "pub fn group_norm(", "pub fn transpose(", "pub fn swish("):
        assert fn in device, fn


def test_ctypes_table_matches_header():
    from any_gpu import _lib
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_status_strings_and_null_handling():
    from any_gpu import _lib
    lib = _lib.load()
    assert lib.agpu_status_string(0) == b"ok"
    assert lib.agpu_status_string(1) == b"shape mismatch"
    assert lib.agpu_status_string(6) == b"device wait timed out"
    # NULL handles are rejected without touching a GPU
    assert lib.agpu_buffer_len(None) == 0
    assert lib.agpu_buffer_free(None) == 0
    assert lib.agpu_synchronize(None) == 2
    assert lib.agpu_set_precision(None, 0) == 2
    out = C.c_void_p()
    assert lib.agpu_matmul(None, None, None, 1, 1, 1, C.byref(out)) == 2
    assert b"NULL" in lib.agpu_last_error_message()
    assert lib.agpu_device_create(0, None) == 2
    assert lib.agpu_selftest_wait_timeout(None, 1000, None) == 2


def test_thread_precision_override_is_thread_local():
    import threading
    from any_gpu import _lib
    lib = _lib.load()
    assert lib.agpu_get_thread_precision() == -1
    assert lib.agpu_set_thread_precision(5) == 2
    assert lib.agpu_set_thread_precision(1) == 0
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.agpu_get_thread_precision()))
    t.start()
    t.join()
    assert lib.agpu_get_thread_precision() == 1 and seen == [-1]
    assert lib.agpu_set_thread_precision(-1) == 0
    assert lib.agpu_get_thread_precision() == -1


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU path")
def test_device_create_without_gpu_reports_no_device():
    from any_gpu import AnyGpuError, GpuDevice
    with pytest.raises(AnyGpuError) as e:
        GpuDevice.gpu(0)
    assert e.value.status == 5


def test_product_does_not_reference_oracle():
    # the shipped package and CUDA sources never import or link the oracle
    for p in list((ROOT / "any-gpu_b200").rglob("*.py")) + list(
            (ROOT / "any-gpu_b200" / "csrc").glob("*.cu*")):
        text = p.read_text()
        assert "oracle" not in text.lower().replace("oracle-free", ""), p


def test_every_environment_switch_is_documented():
    # the kernel-choice switches the library reads are listed in the header
    read = set()
    for p in (ROOT / "any-gpu_b200" / "csrc").glob("*.cu*"):
        read |= set(re.findall(r'getenv\("(AGPU_[A-Z0-9_]+)"\)', p.read_text()))
    documented = set()
    for h in HEADERS:
        documented |= set(re.findall(r"\b(AGPU_[A-Z0-9_]+)=", h.read_text()))
    assert read, "no switches found"
    assert read <= documented, sorted(read - documented)
