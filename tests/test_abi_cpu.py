"""CPU-side checks of the C ABI library: it builds, loads, and exports every
symbol include/prism_b200.h declares.  No compute calls (no GPU here)."""
import ctypes
import os
import subprocess

import pytest

import prism_b200


def test_library_exports_every_header_symbol():
    L = prism_b200.load()
    names = prism_b200.exported_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_library_is_sm100a_only_and_has_no_torch_dependency():
    import build
    lib = prism_b200.LIB_PATH
    out = subprocess.run(["ldd", lib], capture_output=True, text=True).stdout
    deps = [line.split()[0] for line in out.splitlines() if line.strip()]
    assert not [d for d in deps if "torch" in d or d.startswith("libc10")], deps
    # one target: sm_100a, no PTX fallback for other architectures
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = prism_b200.load().prism_b200_executor_create(0, ctypes.byref(h))
    assert st == prism_b200.E_DEVICE and not h.value


def test_supports_is_geometry_only():
    L = prism_b200.load()
    ok = prism_b200.Tensor(35, 4096, 4096, __import__("numpy").zeros(1, "u1"))
    # supports() needs no device: a NULL executor is simply "not eligible"
    assert L.prism_b200_executor_supports(None, ctypes.byref(ok._c())) == 0


@pytest.mark.parametrize("kind", [35, 10])
def test_host_generator_matches_library_generator(kind):
    """The benchmark's reference arm builds its weights with the oracle's
    restatement of the seeded generator, so it never maps the product
    library; both must give the same bytes."""
    import numpy as np
    from oracle import oracle
    for rows, cols, seed, stream in [(7, 512, 0, 0), (33, 2560, 5, 123456), (3, 9216, 1, 7)]:
        a = oracle.synth_weights(kind, rows, cols, seed, stream)
        b = prism_b200.synth_weights(kind, rows, cols, seed, stream)
        assert np.array_equal(a, b), (rows, cols, seed, stream)
