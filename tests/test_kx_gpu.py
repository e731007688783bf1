"""GPU parity of the session key agreement: the device kernel behind
``secure_infer_aicpu_key_agreement_do`` (key_agreement.aicpu) against the CPU
oracle, and ``secure_infer_session_init_key_agreement`` (secure_infer.cpp:
449-521) carrying a reload round trip with the agreed key."""
from __future__ import annotations

import ctypes as ct

import pytest

from conftest import det_bytes
from oracle import kx_oracle as kxo

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import _native
    return _native.lib()


def dev(data: bytes):
    return torch.tensor(list(data), dtype=torch.uint8, device="cuda")


def run_device(lib, host_public: bytes, challenge: bytes):
    hp, ch = dev(host_public), dev(challenge)
    key = torch.zeros(16, dtype=torch.uint8, device="cuda")
    dp = torch.zeros(32, dtype=torch.uint8, device="cuda")
    proof = torch.zeros(32, dtype=torch.uint8, device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = [ct.c_void_p(t.data_ptr()) for t in (hp, ch, key, dp, proof, status)]
    assert lib.secure_infer_aicpu_key_agreement_do(s, *p) == 0
    torch.cuda.synchronize()
    return (bytes(key.cpu().tolist()), bytes(dp.cpu().tolist()), bytes(proof.cpu().tolist()),
            int(status.item()))


def test_device_half_matches_oracle(lib):
    publics = set()
    for i in range(4):
        host_secret, challenge = det_bytes(f"kx-host-{i}", 32), det_bytes(f"kx-challenge-{i}", 32)
        host_public = kxo.x25519_public(host_secret)
        key, dev_public, proof, status = run_device(lib, host_public, challenge)
        assert status == 0
        shared = kxo.x25519(host_secret, dev_public)
        assert shared != bytes(32)
        assert key == kxo.derive_key(shared, host_public, dev_public, challenge)
        assert proof == kxo.derive_proof(key, challenge)
        assert kxo.host_side(host_secret, challenge, dev_public, proof) == (key, kxo.derive_salt(shared))
        publics.add(dev_public)
    assert len(publics) == 4          # a fresh device secret per call


@pytest.mark.parametrize("u", [0, 1])
def test_low_order_host_public_refused(lib, u):
    """A low-order host point gives a zero shared value: the device stops
    with status 2 and writes no key or proof (key_agreement.aicpu:31-34)."""
    key, dev_public, proof, status = run_device(lib, u.to_bytes(32, "little"), det_bytes("kx-c", 32))
    assert status == 2
    assert key == bytes(16) and proof == bytes(32)
    assert dev_public != bytes(32)


def test_session_from_key_agreement_round_trip(lib):
    """Records encrypted by the host with its derived key are verified and
    decrypted by the device with the device's own copy of the key: both ends
    agreed on key and salt."""
    from secure_infer_b200 import native_layerwise as nl
    session = nl.Session.key_agreement(0)
    try:
        heads, blocks, n, layer = 2, 6, 4, 1
        g = torch.Generator().manual_seed(5)
        host = [torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).pin_memory()
                for _ in range(2)]
        for k in range(2):
            nl.register_host_range(host[k], layer, k)
        cache = [torch.zeros((blocks + 2, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        src_ids = torch.tensor([3, 0, 5, 1])
        dst_ids = torch.tensor([7, 2, 0, 4])
        t = nl.NativeTransfer("none", layers=4)
        t.layer = layer
        t.single_layer_kv_transfer((host, torch.stack((src_ids, dst_ids), 1)), cache)
        t.wait_for_layer_load(layer)
        torch.cuda.synchronize()
        for k in range(2):
            assert torch.equal(cache[k].cpu()[dst_ids], host[k][src_ids])
        assert nl.auth_stats()["rejected"] == 0
    finally:
        session.close()
