"""GPU parity of the pre-encryption lookahead (secure_infer_h2d_prepare_layer).

An announced reload is encrypted ahead of time and the matching reload call
copies the prepared records: the result must equal the inline path's (raw
blocks, and codec packets decoded like the reference's decode_into), the
prefetch stats must count what was taken, waited for or missed, and the
session's tamper / strict-retry, invalidation and pool-cap behaviour must
hold for prepared records too."""
from __future__ import annotations

import ctypes as ct
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import det_bytes, load_codec

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
KEY = det_bytes("prepare-key", 16)
SALT = det_bytes("prepare-salt", 4)


@pytest.fixture(scope="module")
def nl():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield native_layerwise
    s.close()


def layer_inputs(nl, heads, blocks, layer, seed):
    g = torch.Generator().manual_seed(seed)
    host = [torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).pin_memory() for _ in range(2)]
    for k in range(2):
        nl.register_host_range(host[k], layer, k)
    cache = [torch.zeros((blocks + 4, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    perm = torch.randperm(blocks + 4, generator=g)[:blocks]
    src = torch.randperm(blocks, generator=g)
    return host, cache, torch.stack((src, perm), 1)


def check(host, cache, mapping):
    torch.cuda.synchronize()
    for k in range(2):
        assert torch.equal(cache[k].cpu()[mapping[:, 1]], host[k][mapping[:, 0]]), k


def test_prepare_then_reload_raw(nl):
    heads, blocks, layer = 4, 10, 2
    host, cache, mapping = layer_inputs(nl, heads, blocks, layer, 1)
    t = nl.NativeTransfer("none", layers=8)
    t.layer = layer
    before = nl.prefetch_stats()
    assert t.prepare_layer((host, mapping), heads)
    assert not t.prepare_layer((host, mapping), heads)       # the same announcement is pending
    t.single_layer_kv_transfer((host, mapping), cache)
    t.wait_for_layer_load(layer)
    check(host, cache, mapping)
    after = nl.prefetch_stats()
    assert after["ready"] - before["ready"] == 2 * blocks
    assert after["missing"] == before["missing"]


@pytest.mark.parametrize("bits", [8, 4])
def test_prepare_codec_kv_pair(nl, bits):
    """Prepared K+V codec packets decode bit-exact like decode_into."""
    heads = 2
    g = load_codec(heads)
    layer = 2 if bits == 8 else 21
    lib = nl._native.lib()
    dst_idx = [int(i) for i in g["dst_idx"]]
    dest = [torch.zeros((6, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    packets, srcs, dsts = [], [], []
    for kind in range(2):
        pk = torch.from_numpy(g[f"packet_k{kind}_b{bits}"]).pin_memory()
        nl.register_host_range(pk, layer, kind)
        packets.append(pk)
        b, width = pk.shape
        srcs += [pk.data_ptr() + i * width for i in range(b)]
        dsts += [dest[kind].data_ptr() + i * dest[kind].stride(0) * 2 for i in dst_idx]
    codec = nl._native.Codec(bits, nl._native.KIND_KV, heads, layer)
    before = nl.prefetch_stats()
    assert lib.secure_infer_h2d_prepare_layer(layer, nl._ptrs(srcs), len(srcs), width, ct.byref(codec)) == 0
    assert lib.secure_infer_h2d_reload_layer(layer, nl._ptrs(srcs), nl._ptrs(dsts), len(srcs), width,
                                             ct.byref(codec), 0, None, nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == 0
    for kind in range(2):
        got = dest[kind].view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got[dst_idx], g[f"dest_k{kind}_b{bits}"]), kind
    assert nl.prefetch_stats()["ready"] - before["ready"] == len(srcs)


def test_prepare_mismatch_and_invalidate(nl):
    """A reload whose sources differ from the announcement encrypts inline
    and counts a miss; invalidation drops the pending entry."""
    heads, blocks, layer = 2, 6, 3
    host, cache, mapping = layer_inputs(nl, heads, blocks, layer, 2)
    other = torch.stack((mapping[:, 0].flip(0), mapping[:, 1]), 1)
    t = nl.NativeTransfer("none", layers=8)
    before = nl.prefetch_stats()
    assert t.prepare_layer((host, mapping), heads, layer=layer)
    t.layer = layer
    t.single_layer_kv_transfer((host, other), cache)
    t.wait_for_layer_load(layer)
    check(host, cache, other)
    mid = nl.prefetch_stats()
    assert mid["missing"] - before["missing"] == 1 and mid["ready"] == before["ready"]
    nl._native.lib().secure_infer_invalidate_transfer_prefetches()
    t.layer = layer
    t.single_layer_kv_transfer((host, mapping), cache)      # nothing pending: inline, no miss
    t.wait_for_layer_load(layer)
    check(host, cache, mapping)
    after = nl.prefetch_stats()
    assert after["missing"] == mid["missing"] and after["ready"] == mid["ready"]


def test_prepare_tamper_then_strict_retry(nl):
    """A byte flipped in a prepared record is rejected; the strict retry
    re-encrypts that record inline with a fresh ticket."""
    heads, blocks, layer = 2, 5, 6
    host, cache, mapping = layer_inputs(nl, heads, blocks, layer, 3)
    t = nl.NativeTransfer("none", layers=8)
    t.layer = layer
    assert t.prepare_layer((host, mapping), heads)
    before = nl.auth_stats()
    nl._native.lib().secure_infer_arm_tamper(1, 4, 0)
    t.single_layer_kv_transfer((host, mapping), cache)
    t.wait_for_layer_load(layer)
    after = nl.auth_stats()
    assert after["rejected"] - before["rejected"] == 1 and after["retried"] - before["retried"] == 1
    check(host, cache, mapping)


def test_prepare_lookahead_pipeline(nl):
    """Each layer's reload is announced while the previous layer reloads."""
    heads, blocks, layers = 8, 6, 5
    inputs = [layer_inputs(nl, heads, blocks, 10 + layer, 20 + layer) for layer in range(layers)]
    t = nl.NativeTransfer("none", layers=32)
    t.layer = 10
    before = nl.prefetch_stats()
    for layer in range(layers):
        host, cache, mapping = inputs[layer]
        if layer + 1 < layers:
            nhost, _, nmap = inputs[layer + 1]
            assert t.prepare_layer((nhost, nmap), heads, layer=t.layer + 1)
        t.single_layer_kv_transfer((host, mapping), cache)
    for layer in range(layers):
        t.wait_for_layer_load(10 + layer)
        check(*inputs[layer])
    assert nl.prefetch_stats()["ready"] - before["ready"] == (layers - 1) * 2 * blocks


CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from secure_infer_b200 import native_layerwise as nl
s = nl.Session(0, bytes(range(16)), bytes([1, 2, 3, 4]))
big = [torch.zeros((4, 128, 8, 128), dtype=torch.bfloat16).pin_memory() for _ in range(2)]      # 2 MiB of records
small = [torch.zeros((1, 128, 4, 128), dtype=torch.bfloat16).pin_memory() for _ in range(2)]   # 256 KiB
t = nl.NativeTransfer("none", layers=4)
m4 = torch.stack((torch.arange(4), torch.arange(4)), 1)
m1 = torch.stack((torch.arange(1), torch.arange(1)), 1)
assert not t.prepare_layer((big, m4), 8, layer=0)
assert t.prepare_layer((small, m1), 4, layer=1)
s.close()
print("cap ok")
"""


def test_prepare_pool_cap():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ, SECURE_INFER_PREPARE_POOL_BYTES=str(1 << 20))
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "cap ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_process_exit_without_shutdown_is_clean(nl):
    """A process that announced a reload (starting the lookahead encryption
    thread) and exits without secure_infer_session_shutdown ends normally,
    instead of std::terminate from a joinable library thread."""
    import subprocess
    import sys
    import textwrap
    from conftest import ROOT
    code = textwrap.dedent("""
        import torch
        from secure_infer_b200 import native_layerwise as nl
        s = nl.Session(0, bytes(range(16)), bytes(4))
        host = torch.zeros((4, 128, 1, 128), dtype=torch.bfloat16).pin_memory()
        nl.register_host_range(host, 3, 0)
        mapping = torch.tensor([[0, 0], [1, 1]])
        t = nl.NativeTransfer("none", layers=4, heads=1)
        assert t.prepare_layer(([host, host], mapping), 1, layer=3)
        print("exiting")
    """)
    out = subprocess.run([sys.executable, "-c", code], cwd=str(ROOT), capture_output=True, text=True, timeout=300,
                         env={**__import__("os").environ, "PYTHONPATH": str(ROOT)})
    assert out.returncode == 0, out.stderr[-2000:]
    assert "exiting" in out.stdout
