"""The C ABI: the library loads without a GPU and exports every entry point include/*.h declares,
and the Python declarations cover exactly those entry points. No compute calls here."""

import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for path in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(telmo_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    from telmo_b200 import _lib
    lib = _lib.load()
    names = declared()
    assert len(names) >= 20
    for name in sorted(names):
        assert hasattr(lib, name), name


def test_python_declarations_match_the_header():
    from telmo_b200 import _lib
    assert set(_lib.SIGNATURES) == declared()


def test_context_creation_without_a_gpu_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        return
    from telmo_b200 import _lib
    h = ctypes.c_void_p()
    rc = _lib.load().telmo_ctx_create(0, ctypes.byref(h))
    assert rc != 0 and not h.value
    assert _lib.load().telmo_last_error(None)


def test_argument_checks_run_before_any_device_work():
    from telmo_b200 import _lib
    L = _lib.load()
    assert L.telmo_ctx_check(None, None) == _lib.TELMO_ERR_ARGUMENT
    assert L.telmo_logmel_rows(0, 16000) == 50
    assert L.telmo_logmel_rows(0, 16160) == 51
    assert L.telmo_logmel_rows(0, 319) == 0
    assert L.telmo_logmel_rows(1, 16000) == 100
