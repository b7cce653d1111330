"""The C ABI without a GPU: the library loads, exports every entry point
include/*.h declare, and rejects bad tensors with the
reference's error texts before it touches a device."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest


def test_exports_every_declared_symbol(wb):
    lib = wb._lib.lib()
    declared = wb._lib.exported_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.wc_version().startswith(b"whistle_b200 ")


def test_no_oracle_in_product(wb):
    """The product library links no oracle symbol and the package imports no
    oracle module."""
    import subprocess
    import sys

    syms = subprocess.run(["nm", "-D", str(wb.LIB_PATH)], capture_output=True, text=True).stdout
    assert "wo_" not in syms
    for name, mod in list(sys.modules.items()):
        if name.startswith("go-whistle_b200"):
            src = getattr(mod, "__file__", "") or ""
            if src.endswith(".py"):
                assert "import oracle" not in open(src).read(), name


def _good(wb):
    rng = np.random.default_rng(7)
    return wb.synth.random_packed(rng, 2, 128, 128, 2, "reference")


# internal/cq/cq_test.go:561 TestNewErrors
NEW_ERRORS = [
    ("3 bits", lambda p: (setattr(p, "Bits", 3), setattr(p, "Width", 3)), "not supported"),
    ("ternary", lambda p: setattr(p, "Bits", 5), "not supported"),
    ("group 24", lambda p: setattr(p, "Group", 24), "power of two"),
    ("codebook", lambda p: setattr(p, "Codebook", p.Codebook[:3]), "codebook"),
    ("index", lambda p: setattr(p, "Index", p.Index[1:]), "index"),
    ("norms", lambda p: setattr(p, "Norms", p.Norms[2:]), "norm"),
]


@pytest.mark.parametrize("name,edit,want", NEW_ERRORS, ids=[c[0] for c in NEW_ERRORS])
def test_new_errors(wb, name, edit, want):
    p = _good(wb)
    edit(p)
    with pytest.raises(wb.CQError) as e:
        wb.cq.New(p)
    assert want in str(e.value)
    assert str(e.value).startswith("cq: ")


def test_error_messages_match_reference(wb):
    p = _good(wb)
    p.Group = 24
    with pytest.raises(wb.CQError, match=r"^cq: group 24 is not a power of two >= 8$"):
        wb.cq.New(p)
    p = _good(wb)
    p.Index = p.Index[1:]
    with pytest.raises(wb.CQError, match=r"^cq: 63 index and 4 norm bytes for \[2, 128\], want 64 and 4$"):
        wb.cq.New(p)


def test_null_arguments(wb):
    lib = wb._lib.lib()
    assert lib.wc_cq_create(None, 0, None, 0, None, 0, 1, 8, 8, 2, 2, None) == wb._lib.WC_ERR_INVALID
    v = ctypes.c_void_p()
    assert lib.wc_cq_rows(None, 0, 0, ctypes.byref(v)) == wb._lib.WC_ERR_INVALID
    assert lib.wc_cq_gemm(None, None, None, 1, None) == wb._lib.WC_ERR_INVALID
    assert "nil" in wb._lib.last_error()
    assert lib.wc_quantize_rows(None, 1, 96, 40, None, None, None) == wb._lib.WC_ERR_INVALID
    assert wb._lib.last_error() == "needle: int8 rows of 96 in chunks of 40"
    assert lib.wc_attend_int8(None, 1, 8, None, None, None, None, 3, 3, 48, 64, None, 1.0, 1, None, None,
                              None) == wb._lib.WC_ERR_INVALID


def test_int8rows_panics(wb):
    """int8_test.go:128-141: bad chunking and partial rows panic."""
    with pytest.raises(wb.Panic):
        wb.needle.NewInt8Rows(96, 40)
    with pytest.raises(wb.Panic):
        wb.needle.NewInt8Rows(96, 48).Append(np.zeros(50, np.float32))
    assert wb.needle.Int8Rows(0, 1).Len() == 0
