"""The C-ABI library loads without a GPU and exports every symbol include/pk.h declares."""
import os
import re

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


def test_library_is_in_tree_and_sm100a(pk):
    assert pk.LIB_PATH.startswith(ROOT)
    data = open(pk.LIB_PATH, "rb").read()
    assert b"sm_100a" in data


def test_product_library_does_not_link_the_oracle(pk):
    data = open(pk.LIB_PATH, "rb").read()
    assert b"pko_" not in data and b"pk_oracle" not in data
