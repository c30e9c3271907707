"""CPU checks of the drop-in boundary: the C-ABI library builds, loads without a GPU, exports every
symbol include/sa3k.h declares, and refuses to run without an sm_100 device (no CPU fallback)."""
import ctypes
import os
import re

import sa3k

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(REPO, "include", "sa3k.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sa3k_[a-z0-9_]+)\s*\(", txt)))


def test_header_and_binding_agree():
    assert sorted(sa3k.ABI_SYMBOLS) == declared_symbols()


def test_library_exports_every_declared_symbol(sa3k_lib):
    for name in declared_symbols():
        assert hasattr(sa3k_lib, name), name


def test_version_string(sa3k_lib):
    assert b"sm_100a" in sa3k_lib.sa3k_version()


def test_no_cpu_fallback_without_device(sa3k_lib):
    import torch
    if torch.cuda.is_available():
        return
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    rc = sa3k_lib.sa3k_ctx_create(0, ctypes.byref(h), err, 256)
    assert rc != 0 and b"no CUDA device" in err.value
