"""The C-ABI library loads without a GPU and exports every symbol include/pk.h declares."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "pk.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(pk_[a-z0-9_]+)\s*\(", text))
    names.discard("pk_token_cb")  # typedef of a callback, not an export
    return names


def test_header_declares_expected_surface():
    names = declared_functions()
    for must in ("pk_q8_quantize", "pk_matmul", "pk_backend_matvec", "pk_generate", "pk_forward", "pk_logits"):
        assert must in names


def test_library_exports_every_declared_symbol(pk):
    lib = pk.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header(pk):
    assert declared_functions() == set(pk.SYMBOLS)


def test_host_only_entry_points_work_without_gpu(pk):
    lib = pk.lib()
    assert lib.pk_version() >= 100
    for t, want in ((12, 1), (14, 1), (2, 1), (8, 1), (0, 0), (1, 0), (10, 0), (11, 0), (13, 0)):
        assert lib.pk_supports(t) == want, t
    assert pk.packed_bytes(pk.Q6_K, 2304, 16) >= 16 * 9 * 210
    assert pk.packed_bytes(pk.Q4_K, 2304, 16) == 16 * 9 * 144
    assert pk.packed_bytes(pk.Q8_0, 5760, 2) >= 2 * 180 * 34
    assert pk.packed_bytes(3, 64, 1) == 0  # Q4_1 is not a device matvec type


def test_library_is_in_tree(pk):
    assert pk.LIB_PATH.startswith(ROOT)


def test_product_library_does_not_link_the_oracle(pk):
    """Exported symbols and the dynamic section only: no oracle function is
    defined in the product library and it does not load the oracle's."""
    nm = subprocess.run(["nm", "-D", "--defined-only", pk.LIB_PATH], capture_output=True, text=True, check=True)
    names = [ln.split()[-1] for ln in nm.stdout.splitlines() if ln.strip()]
    assert any(n.startswith("pk_") for n in names)
    assert not [n for n in names if n.startswith("pko_")]
    dyn = subprocess.run(["readelf", "-d", pk.LIB_PATH], capture_output=True, text=True, check=True).stdout
    needed = [ln for ln in dyn.splitlines() if "(NEEDED)" in ln]
    assert needed and not [ln for ln in needed if "oracle" in ln]


@pytest.mark.gpu
def test_device_code_is_sm100a(pk):
    """The kernels CUDA loads on the device are sm_100a binaries (no PTX JIT)."""
    import ctypes

    v = ctypes.c_int(0)
    pk._check(pk.lib().pk_device_binary_version(ctypes.byref(v)))
    assert v.value == 100
