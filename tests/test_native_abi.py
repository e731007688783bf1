"""The C-ABI library loads and exports every function include/*.h declares (no GPU)."""
from __future__ import annotations

import re

from conftest import ROOT


def declared_functions() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(secure_infer_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    from secure_infer_b200 import _native
    lib = _native.lib()
    declared = declared_functions()
    assert declared, "no declarations found"
    missing = sorted(n for n in declared if not hasattr(lib, n))
    assert not missing, missing


def test_python_signatures_cover_declarations():
    from secure_infer_b200 import _native
    bound = set(_native.PLUGIN_SIGNATURES) | set(_native.HOST_SIGNATURES)
    assert declared_functions() <= bound


def test_kernel_profile_names_and_empty_collect():
    """The kernel profile entry points work without a GPU when nothing ran."""
    import ctypes as ct
    from secure_infer_b200 import _native
    lib = _native.lib()
    names = []
    k = 0
    while (name := lib.secure_infer_kernel_name(k)) is not None:
        names.append(name.decode())
        k += 1
    assert {"gcm_layer_ctr_kernel", "gcm_layer_verify_kernel", "gcm_layer_encrypt", "kv_encode_kernel"} <= set(names)
    us = (ct.c_double * len(names))()
    cnt = (ct.c_uint64 * len(names))()
    assert lib.secure_infer_kernel_profile_collect(us, cnt, len(names)) == 0
    assert list(cnt) == [0] * len(names)
