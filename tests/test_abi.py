"""The C-ABI library loads without a GPU and exports exactly what
include/ds3_cuda.h declares; host-side validation works before any device
call. No compute runs here."""

from __future__ import annotations

import ctypes as C
import subprocess

import pytest

from qw3_b200 import build, ds3


@pytest.fixture(scope="module")
def lib():
    build.build()
    return ds3.lib()


def exported(path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}


def test_every_declared_symbol_is_exported(lib):
    declared = set(ds3.header_symbols())
    assert len(declared) >= 40
    syms = exported(ds3.LIB_PATH)
    missing = declared - syms
    assert not missing, f"declared but not exported: {sorted(missing)}"
    extra = {s for s in syms if s.startswith("ds3_cuda_")} - declared
    assert not extra, f"exported but not declared: {sorted(extra)}"


def test_python_mirror_covers_the_header(lib):
    declared = {s[len("ds3_cuda_"):] for s in ds3.header_symbols()}
    assert declared == set(ds3._SIGS), declared ^ set(ds3._SIGS)


def test_build_targets_only_sm100a():
    # The build asks nvcc for sm_100a machine code and nothing else (no PTX
    # for JIT, no other architecture); the GPU suite checks the loaded
    # kernels' binary version at run time.
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_calls_before_init_fail_cleanly(lib):
    # No device in this container (or init not called): every op returns -1,
    # allocators return NULL, nothing crashes.
    assert lib.ds3_cuda_rms_norm(None, None, None, 128, 1, C.c_float(1e-6)) == -1
    assert lib.ds3_cuda_buffer_alloc(1024) is None
    assert lib.ds3_cuda_begin_batch() == -1
    assert "not initialised" in ds3.last_error()
    assert lib.ds3_cuda_buffer_wrap(None, 16) is None
    v = lib.ds3_cuda_buffer_wrap(C.c_void_p(0x1000), 64)
    assert v and lib.ds3_cuda_buffer_size(v) == 64
    sub = lib.ds3_cuda_buffer_view(v, 16, 32)
    assert sub and lib.ds3_cuda_buffer_device_ptr(sub) == 0x1010
    assert lib.ds3_cuda_buffer_view(v, 48, 32) is None
    lib.ds3_cuda_buffer_free(sub)
    lib.ds3_cuda_buffer_free(v)


def test_init_without_gpu_reports_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert ds3.init() == -1
    assert "device" in ds3.last_error()
