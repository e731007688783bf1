"""GPU parity of the bitsliced AES keystream kernel (gcm_layer_ctr_bs_kernel,
selected with SECURE_INFER_AES_KEYSTREAM=bitsliced) against the T-table
keystream kernel and the oracle, through secure_infer_keystream_records and a
full device reload."""
from __future__ import annotations

import ctypes as ct
import os
import struct

import pytest

from conftest import det_bytes
from oracle import gcm as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("bs-gpu-key", 16)
SALT = det_bytes("bs-gpu-salt", 4)


@pytest.fixture(scope="module")
def nl():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield native_layerwise
    s.close()
    os.environ.pop("SECURE_INFER_AES_KEYSTREAM", None)


def keystream(nl, tickets, count, variant):
    lib = nl._native.lib()
    n = len(tickets)
    stride = (count + 15) // 16 * 16 + 16
    ks = torch.full((n * stride,), 0xEE, dtype=torch.uint8, device="cuda")
    os.environ["SECURE_INFER_AES_KEYSTREAM"] = variant
    try:
        assert lib.secure_infer_keystream_records((ct.c_uint64 * n)(*tickets), n, count, ks.data_ptr(),
                                                  nl._stream()) == 0
        torch.cuda.synchronize()
    finally:
        os.environ.pop("SECURE_INFER_AES_KEYSTREAM", None)
    return ks.cpu().numpy().reshape(n, stride)


@pytest.mark.parametrize("count,n", [(262144, 3), (16, 5), (1000, 7), (10256, 130), (4096 * 16 + 5, 2)])
def test_bitsliced_keystream_equals_ttable_and_oracle(nl, count, n):
    tickets = [int.from_bytes(det_bytes(f"t{count}.{i}", 6), "big") + 1 for i in range(n)]
    bs = keystream(nl, tickets, count, "bitsliced")
    tt = keystream(nl, tickets, count, "ttable")
    assert (bs == tt).all()
    stride = bs.shape[1]
    for i in (0, n - 1):
        iv = list(struct.unpack(">III", SALT + tickets[i].to_bytes(8, "big"))) + [2]
        want = orc.keystream(KEY, (count + 15) // 16 * 16, iv)
        assert bs[i, :len(want)].tobytes() == want
        j0 = SALT + tickets[i].to_bytes(8, "big") + struct.pack(">I", 1)
        assert bs[i, stride - 16:].tobytes() == orc.aes_block(KEY, j0)


def test_reload_with_bitsliced_keystream(nl):
    """A device reload whose keystream comes from the bitsliced kernel lands
    the host plaintext and authenticates every record."""
    lib = nl._native.lib()
    n, count = 6, 262144
    g = torch.Generator().manual_seed(5)
    plain = torch.randint(0, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    stride = nl.record_bytes(count)
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tk = (ct.c_uint64 * n)()
    assert lib.secure_infer_h2d_encrypt_records(nl._ptrs(plain.data_ptr() + i * count for i in range(n)), count, n,
                                                recs.data_ptr(), stride, tk) == 0
    drecs = recs.cuda()
    dest = torch.zeros((n, count), dtype=torch.uint8, device="cuda")
    ks = torch.empty(n * (count + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    os.environ["SECURE_INFER_AES_KEYSTREAM"] = "bitsliced"
    try:
        assert lib.secure_infer_reload_records(4, drecs.data_ptr(), stride, count, n, tk,
                                               nl._ptrs(dest.data_ptr() + i * count for i in range(n)), ks.data_ptr(),
                                               status.data_ptr(), None, nl._stream(), None) == 0
        torch.cuda.synchronize()
    finally:
        os.environ.pop("SECURE_INFER_AES_KEYSTREAM", None)
    assert status.cpu().tolist() == [1] * n
    assert torch.equal(dest.cpu(), plain)
