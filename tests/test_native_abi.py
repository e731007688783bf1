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


def test_preloaded_library_binds_through_process_namespace():
    """With the library LD_PRELOADed (the reference's deployment, run.sh:66),
    the Python side binds its symbols through ctypes.CDLL(None)."""
    import os
    import subprocess
    import sys
    from secure_infer_b200 import _native
    code = ("import sys; sys.path.insert(0, sys.argv[1]); from secure_infer_b200 import _native; "
            "h = _native.lib(); print(h._name, h.secure_infer_record_bytes(100))")
    env = dict(os.environ, LD_PRELOAD=str(_native.LIB_PATH))
    out = subprocess.run([sys.executable, "-c", code, str(ROOT)], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.split() == ["None", str(_native.lib().secure_infer_record_bytes(100))]
