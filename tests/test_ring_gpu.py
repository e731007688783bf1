"""GPU parity of the chunk-ring H2D staging (SECURE_INFER_H2D_RING=1).

The staging settings are read once per process, so each case runs a small
reload in a child process: 2 ring buffers of 64 KiB force one record per
chunk, many chunks per layer and a wait on the ring's previous copy for most
of them.  Bytes must equal the host plaintext, and a flipped ciphertext byte
must be rejected and recovered by the strict retry."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from secure_infer_b200 import native_layerwise as nl
heads, blocks, layer, tamper = int(sys.argv[2]), int(sys.argv[3]), 4, int(sys.argv[4])
s = nl.Session(0, bytes(range(16)), bytes([9, 8, 7, 6]))
g = torch.Generator().manual_seed(heads * 100 + blocks)
host = [torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).pin_memory() for _ in range(2)]
for k in range(2):
    nl.register_host_range(host[k], layer, k)
cache = [torch.zeros((blocks + 3, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
perm = torch.randperm(blocks + 3, generator=g)[:blocks]
mapping = torch.stack((torch.arange(blocks), perm), 1)
lib = nl._native.lib()
if tamper:
    lib.secure_infer_arm_tamper(1, tamper, 0)
t = nl.NativeTransfer("none", layers=8)
for rep in range(3):                      # the ring wraps across calls too
    t.layer = layer
    t.single_layer_kv_transfer((host, mapping), cache)
    t.wait_for_layer_load(layer)
torch.cuda.synchronize()
for k in range(2):
    assert torch.equal(cache[k].cpu()[perm], host[k]), k
st = nl.auth_stats()
assert st["rejected"] == (1 if tamper else 0) and st["retried"] == (1 if tamper else 0), st
s.close()
print("ring ok")
"""


@pytest.mark.parametrize("heads,blocks,tamper", [(2, 12, 0), (8, 9, 5), (1, 40, 0)])
def test_ring_staging_reload(heads, blocks, tamper):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ, SECURE_INFER_H2D_RING="1", SECURE_INFER_H2D_RING_SLOTS="2",
               SECURE_INFER_H2D_RING_CHUNK=str(64 << 10))
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(heads), str(blocks), str(tamper)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ring ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
