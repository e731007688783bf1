"""The opt-in cudaMemcpyAsync interposer (libsecure_infer_interpose.so), the
CUDA form of the reference's interposed vendor copy (secure_infer.cpp:
7729-7855).  Each case runs in a child process started with LD_PRELOAD, the
way the reference's run.sh loads its library."""
from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap

import pytest

from conftest import ROOT

INTERPOSE = ROOT / "secure_infer_b200" / "_build" / "libsecure_infer_interpose.so"


def run_child(code: str, interpose: bool, timeout: int = 300) -> dict:
    if not INTERPOSE.exists():
        pytest.fail(f"{INTERPOSE} is missing; build with `python -m secure_infer_b200.build`")
    env = dict(os.environ, LD_PRELOAD=str(INTERPOSE), SECURE_INFER_INTERPOSE="1" if interpose else "0",
               PYTHONPATH=str(ROOT))
    out = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], env=env, capture_output=True, text=True,
                         timeout=timeout, cwd=str(ROOT))
    assert out.returncode == 0, out.stderr[-3000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


ROUTING = """
import ctypes as ct, json
import numpy as np
proc = ct.CDLL(None)
from secure_infer_b200 import _native
lib = _native.lib()
fn = proc.cudaMemcpyAsync
fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_int, ct.c_void_p]
fn.restype = ct.c_int
host = np.zeros(4096, np.uint8)
other = np.zeros(4096, np.uint8)
lib.secure_infer_register_host_range_ex(host.ctypes.data, host.nbytes, 3, 0, 1024)
res = {
    "bound_to_library": lib._name is None,
    "registered": lib.secure_infer_is_registered_host_range(host.ctypes.data + 1024, 1024),
    "unregistered": lib.secure_infer_is_registered_host_range(other.ctypes.data, 1024),
    "straddling": lib.secure_infer_is_registered_host_range(host.ctypes.data + 3072, 2048),
    # H2D from a registered range with no session: refused, never a plain copy.
    "h2d_registered": fn(other.ctypes.data, host.ctypes.data, 1024, 1, None),
    # D2H into a registered range with no session: refused as well.
    "d2h_registered": fn(host.ctypes.data, other.ctypes.data, 1024, 2, None),
    # Anything else goes to the CUDA runtime (here: no device, so its error).
    "h2d_other": fn(other.ctypes.data, other.ctypes.data, 1024, 1, None),
}
print(json.dumps(res))
"""


def test_interposer_routes_only_registered_copies():
    """Without a GPU: a copy touching a registered range goes to the library
    (which refuses it without a session: cudaErrorInvalidValue = 1), any other
    copy reaches the CUDA runtime (an error other than 1 with no device, 0 with
    one); with SECURE_INFER_INTERPOSE unset, every copy reaches the runtime."""
    on = run_child(ROUTING, interpose=True)
    assert on["bound_to_library"]           # the preloaded library, through ctypes.CDLL(None)
    assert (on["registered"], on["unregistered"], on["straddling"]) == (1, 0, 0)
    assert on["h2d_registered"] == 1 and on["d2h_registered"] == 1
    assert on["h2d_other"] != 1
    off = run_child(ROUTING, interpose=False)
    assert off["h2d_registered"] == off["h2d_other"] != 1


GPU_COPY = """
import ctypes as ct, json
import torch
from secure_infer_b200 import _native, native_layerwise as nl
torch.cuda.set_device(0)
lib = _native.lib()
session = nl.Session(0, bytes(range(16)), b"\\x01\\x02\\x03\\x04")
heads, blocks, layer = 2, 4, 7
g = torch.Generator().manual_seed(3)
host = torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).pin_memory()
nl.register_host_range(host, layer, 0)
plain_host = torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).pin_memory()
dev = torch.zeros((blocks + 2, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
before = nl.auth_stats()
# An unmodified caller: per-block torch copies of the registered host pool
# inside the reference's layer bracket.
table = [4, 0, 3, 2]                  # host block i -> device block table[i]
assert lib.secure_infer_h2d_layer_group_begin(blocks) == 0
for i in range(blocks):
    dev[table[i]].copy_(host[i], non_blocking=True)
assert lib.secure_infer_h2d_layer_group_end() == 0
auth = lib.secure_infer_recovery_wait_layer_authentication(layer)
torch.cuda.synchronize()
after = nl.auth_stats()
ok = all(torch.equal(dev[table[i]].cpu(), host[i]) for i in range(blocks))
# A copy from an unregistered buffer is a plain copy: no new authentications.
dev[blocks + 1].copy_(plain_host[0])
torch.cuda.synchronize()
plain_ok = torch.equal(dev[blocks + 1].cpu(), plain_host[0])
after_plain = nl.auth_stats()
# D2H into a registered host range: device encrypt + tag, host verify.
back = torch.zeros((blocks, 128, heads, 128), dtype=torch.bfloat16).pin_memory()
nl.register_host_range(back, layer, 1)
src = torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).cuda()
for i in range(blocks):
    back[i].copy_(src[i])
wait = lib.secure_infer_d2h_wait()
d2h_ok = torch.equal(back, src.cpu())
session.close()
print(json.dumps({"auth": auth, "verified": after["verified"] - before["verified"], "ok": ok,
                  "plain_ok": plain_ok, "verified_after_plain": after_plain["verified"] - after["verified"],
                  "wait": wait, "d2h_ok": d2h_ok}))
"""


@pytest.mark.gpu
def test_interposed_torch_copies_arrive_authenticated():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    r = run_child(GPU_COPY, interpose=True)
    assert r["auth"] == 0 and r["ok"]
    assert r["verified"] == 4                       # every block went through the verify kernel
    assert r["plain_ok"] and r["verified_after_plain"] == 0
    assert r["wait"] == 0 and r["d2h_ok"]
