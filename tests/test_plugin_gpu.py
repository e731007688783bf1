"""GPU parity of the plugin ABI (GHASH_LIBRARY entry points) against the
reference's own KAT procedure (secure_infer/tests/crypto_smoke.py:39-67) and
the CPU oracle.  Every call goes through the C ABI with device pointers."""
from __future__ import annotations

import ctypes as ct
import struct

import numpy as np
import pytest

from conftest import det_bytes
from oracle import gcm as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FLAGS_FINALIZE, FLAGS_VERIFY, FLAGS_XOR = 1, 2, 4


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import _native
    return _native.lib()


def dev(data: bytes, offset: int = 0):
    """Device copy of `data`, optionally starting `offset` bytes into the allocation."""
    buf = torch.zeros(len(data) + offset + 16, dtype=torch.uint8, device="cuda")
    view = buf[offset:offset + len(data)]
    if data:
        view.copy_(torch.frombuffer(bytearray(data), dtype=torch.uint8))
    return view


def empty(n: int, offset: int = 0):
    buf = torch.full((n + offset + 16,), 0xA5, dtype=torch.uint8, device="cuda")
    return buf[offset:offset + n]


def host(t) -> bytes:
    torch.cuda.synchronize()
    return t.cpu().numpy().tobytes()


def ptr(t):
    return ct.c_void_p(t.data_ptr())


def stream():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def status_buf():
    return torch.full((1,), 7, dtype=torch.int32, device="cuda")


def case_inputs(case):
    key, h = bytes.fromhex(case["key"]), bytes.fromhex(case["h"])
    aad = bytes.fromhex(case["aad"])
    plain = det_bytes(case["plain_seed"], case["count"])
    return key, h, aad, plain, case["iv_words"]


@pytest.mark.parametrize("index", range(4))
def test_crypto_smoke_kat(lib, gcm_kat, index):
    """The reference device KAT: encrypt_tag == AESGCM, decrypt_verify_aad and
    keystream + verify_xor_aad restore the plaintext with status 1."""
    case = gcm_kat[index]
    key, h, aad, plain, iv = case_inputs(case)
    count = len(plain)
    dk, dh, da, src = dev(key), dev(h), dev(aad), dev(plain)
    c_out, tag = empty(count), empty(16)
    assert lib.secure_infer_aicpu_gcm_encrypt_tag_do(stream(), ptr(src), ptr(dk), ptr(dh), ptr(c_out), ptr(tag),
                                                      count, *iv, ptr(da), len(aad)) == 0
    cipher = host(c_out)
    assert host(tag).hex() == case["tag"]
    if "cipher" in case:
        assert cipher.hex() == case["cipher"]
    dc, dt = dev(cipher), dev(bytes.fromhex(case["tag"]))
    restored, st = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt),
                                                             ptr(restored), ptr(st), count, *iv, ptr(da),
                                                             len(aad)) == 0
    assert host(restored) == plain and int(st.item()) == 1
    ks = empty(count)
    assert lib.secure_infer_aicpu_keystream_do(stream(), ptr(dk), ptr(ks), count, *iv) == 0
    assert host(ks) == orc.keystream(key, count, iv)
    restored2, st2 = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_verify_xor_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(ks),
                                                         ptr(restored2), ptr(st2), count, *iv, ptr(da),
                                                         len(aad)) == 0
    assert host(restored2) == plain and int(st2.item()) == 1


@pytest.mark.parametrize("index", range(4))
def test_no_aad_entry_points(lib, gcm_kat, index):
    case = gcm_kat[index]
    key, h, _, plain, iv = case_inputs(case)
    count = len(plain)
    c, tag = orc.gcm_encrypt_tag(plain, key, h, iv, None)
    assert tag.hex() == case["tag_noaad"]
    dk, dh, dc, dt = dev(key), dev(h), dev(c), dev(tag)
    out, st = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_decrypt_verify_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(out),
                                                         ptr(st), count, *iv) == 0
    assert host(out) == plain and int(st.item()) == 1
    ks = dev(orc.keystream(key, count, iv))
    out2, st2 = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_verify_xor_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(ks),
                                                     ptr(out2), ptr(st2), count, *iv) == 0
    assert host(out2) == plain and int(st2.item()) == 1
    st3 = status_buf()
    assert lib.secure_infer_aicpu_gcm_verify_only_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(st3),
                                                      count, *iv) == 0
    assert int(st3.item()) == 1


@pytest.mark.parametrize("count", [16, 31, 4096, 65536 + 5, 262144, 1048576 + 13])
@pytest.mark.parametrize("target", ["cipher", "tag", "aad"])
def test_tamper_rejected_and_zeroed(lib, count, target):
    """A flipped ciphertext/tag/AAD bit gives status 0 and an all-zero output
    (secure_infer.cpp:7170-7189 expectation)."""
    key = det_bytes(f"tk{count}", 16)
    iv = [*struct.unpack(">III", det_bytes(f"tn{count}", 12)), 2]
    aad = det_bytes(f"ta{count}", 64)
    plain = det_bytes(f"tp{count}", count)
    h = orc.aes_block(key, bytes(16))
    c, tag = orc.gcm_encrypt_tag(plain, key, h, iv, aad)
    flip = lambda b, i: b[:i] + bytes([b[i] ^ 0x10]) + b[i + 1:]  # noqa: E731
    if target == "cipher":
        c = flip(c, count // 2)
    elif target == "tag":
        tag = flip(tag, 15)
    else:
        aad = flip(aad, 40)
    dk, dh, dc, dt, da = dev(key), dev(h), dev(c), dev(tag), dev(aad)
    out, st = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(out),
                                                             ptr(st), count, *iv, ptr(da), len(aad)) == 0
    assert int(st.item()) == 0 and host(out) == bytes(count)
    ks = dev(orc.keystream(key, count, iv))
    out2, st2 = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_verify_xor_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(ks),
                                                         ptr(out2), ptr(st2), count, *iv, ptr(da), len(aad)) == 0
    assert int(st2.item()) == 0 and host(out2) == bytes(count)
    st3 = status_buf()
    assert lib.secure_infer_aicpu_gcm_verify_only_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(st3),
                                                          count, *iv, ptr(da), len(aad)) == 0
    assert int(st3.item()) == 0


@pytest.mark.parametrize("count", [1, 17, 64, 4095, 65536 + 5, 131072 - 7, 4 * 1048576 + 3])
@pytest.mark.parametrize("offset", [0, 3])
def test_sizes_and_alignment_vs_oracle(lib, count, offset):
    key = det_bytes(f"sk{count}", 16)
    iv = [*struct.unpack(">III", det_bytes(f"sn{count}", 12)), 0xFFFFFFF0]   # counter wraps
    aad = det_bytes(f"sa{count}", 37)   # AAD not a multiple of 16
    plain = det_bytes(f"sp{count}", count)
    h = orc.aes_block(key, bytes(16))
    c_ref, tag_ref = orc.gcm_encrypt_tag(plain, key, h, iv, aad)
    dk, dh, da = dev(key), dev(h), dev(aad)
    src = dev(plain, offset)
    c_out, tag = empty(count, offset), empty(16)
    assert lib.secure_infer_aicpu_gcm_encrypt_tag_do(stream(), ptr(src), ptr(dk), ptr(dh), ptr(c_out), ptr(tag),
                                                      count, *iv, ptr(da), len(aad)) == 0
    assert host(c_out) == c_ref and host(tag) == tag_ref
    dc, dt = dev(c_ref, offset), dev(tag_ref)
    out, st = empty(count, offset), status_buf()
    assert lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do(stream(), ptr(dc), ptr(dk), ptr(dh), ptr(dt), ptr(out),
                                                             ptr(st), count, *iv, ptr(da), len(aad)) == 0
    assert int(st.item()) == 1 and host(out) == plain
    ctr_out = empty(count, offset)
    assert lib.secure_infer_aicpu_aes_ctr_do(stream(), ptr(src), ptr(dk), ptr(ctr_out), count, *iv) == 0
    assert host(ctr_out) == c_ref


def test_ghash_flags_and_auth_gate(lib, gcm_kat):
    case = gcm_kat[2]
    key, h, aad, plain, iv = case_inputs(case)
    count = len(plain)
    c, tag = orc.gcm_encrypt_tag(plain, key, h, iv, aad)
    mask = orc.keystream(key, 16, iv[:3] + [1])
    ks = orc.keystream(key, count, iv)
    dc, dh, da, dm, dt, dks = dev(c), dev(h), dev(aad), dev(mask), dev(tag), dev(ks)
    out16, plain_out, st = empty(16), empty(count), status_buf()
    assert lib.secure_infer_aicpu_ghash_do(stream(), ptr(dc), ptr(dh), ptr(out16), ptr(da), ptr(dm), ptr(dt),
                                           ptr(dks), ptr(plain_out), ptr(st), count, len(aad),
                                           FLAGS_FINALIZE | FLAGS_VERIFY | FLAGS_XOR) == 0
    assert host(out16) == tag and int(st.item()) == 1 and host(plain_out) == plain
    # Raw GHASH without mask, verify, or XOR; no status pointer.
    out16b = empty(16)
    assert lib.secure_infer_aicpu_ghash_do(stream(), ptr(dc), ptr(dh), ptr(out16b), ptr(da), None, None, None,
                                           None, None, count, len(aad), 0) == 0
    assert host(out16b) == orc.ghash(h, aad, c)
    # Wrong expected tag: status 0 and the XOR output is withheld.
    bad = dev(bytes(16))
    plain_bad, st_bad = empty(count), status_buf()
    assert lib.secure_infer_aicpu_ghash_do(stream(), ptr(dc), ptr(dh), ptr(out16), ptr(da), ptr(dm), ptr(bad),
                                           ptr(dks), ptr(plain_bad), ptr(st_bad), count, len(aad),
                                           FLAGS_FINALIZE | FLAGS_VERIFY | FLAGS_XOR) == 0
    assert int(st_bad.item()) == 0 and host(plain_bad) == bytes(count)
    # auth_gate: status 1 keeps, anything else zeroes.
    data = dev(plain)
    ok = torch.ones(1, dtype=torch.int32, device="cuda")
    assert lib.secure_infer_aicpu_auth_gate_do(stream(), ptr(data), ptr(ok), count) == 0
    assert host(data) == plain
    no = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.secure_infer_aicpu_auth_gate_do(stream(), ptr(data), ptr(no), count) == 0
    assert host(data) == bytes(count)


def test_batches_and_xor_only(lib):
    key = det_bytes("bk", 16)
    h = orc.aes_block(key, bytes(16))
    count = 262144
    n = 4
    ivs = [[*struct.unpack(">III", det_bytes(f"bn{i}", 12)), 2] for i in range(n)]
    aads = [det_bytes(f"ba{i}", 64) for i in range(n)]
    plains = [det_bytes(f"bp{i}", count) for i in range(n)]
    enc = [orc.gcm_encrypt_tag(p, key, h, iv, a) for p, iv, a in zip(plains, ivs, aads)]
    dk, dh = dev(key), dev(h)
    # keystream_batch (32-entry descriptor max; use 7 entries)
    outs = [empty(count) for _ in range(7)]
    iv_arr = (ct.c_uint32 * 28)(*[w for i in range(7) for w in ivs[i % n][:3] + [2 + i]])
    ptrs = (ct.c_void_p * 7)(*[o.data_ptr() for o in outs])
    assert lib.secure_infer_aicpu_keystream_batch_do(stream(), ptr(dk), ptrs, iv_arr, count, 7) == 0
    for i in range(7):
        assert host(outs[i]) == orc.keystream(key, count, ivs[i % n][:3] + [2 + i])
    assert lib.secure_infer_aicpu_keystream_batch_do(stream(), ptr(dk), ptrs, iv_arr, count, 33) == -1
    # verify_xor_batch with record 2 tampered
    cs = [dev(c if i != 2 else bytes([c[0] ^ 1]) + c[1:]) for i, (c, _) in enumerate(enc)]
    tags = [dev(t) for _, t in enc]
    kss = [dev(orc.keystream(key, count, iv)) for iv in ivs]
    douts = [empty(count) for _ in range(n)]
    sts = [status_buf() for _ in range(n)]
    da = [dev(a) for a in aads]
    arr = lambda ts: (ct.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
    iv4 = (ct.c_uint32 * (4 * n))(*[w for iv in ivs for w in iv])
    assert lib.secure_infer_aicpu_gcm_verify_xor_batch_do(stream(), ptr(dk), ptr(dh), arr(cs), arr(tags), arr(kss),
                                                          arr(douts), arr(sts), arr(da), count, 64, iv4, n) == 0
    for i in range(n):
        if i == 2:
            assert int(sts[i].item()) == 0 and host(douts[i]) == bytes(count)
        else:
            assert int(sts[i].item()) == 1 and host(douts[i]) == plains[i]
    # xor_only: no authentication, status forced to 1
    xo, st = empty(count), status_buf()
    assert lib.secure_infer_aicpu_gcm_xor_only_do(stream(), ptr(cs[2]), ptr(dk), ptr(dh), ptr(tags[2]), ptr(kss[2]),
                                                  ptr(xo), ptr(st), count, *ivs[2]) == 0
    c2 = bytes([enc[2][0][0] ^ 1]) + enc[2][0][1:]
    assert int(st.item()) == 1 and host(xo) == bytes(a ^ b for a, b in zip(c2, orc.keystream(key, count, ivs[2])))


def test_null_and_zero_arguments_rejected(lib):
    t = empty(32)
    assert lib.secure_infer_aicpu_keystream_do(stream(), None, ptr(t), 32, 0, 0, 0, 2) == -1
    assert lib.secure_infer_aicpu_keystream_do(stream(), ptr(t), ptr(t), 0, 0, 0, 0, 2) == -1
    assert lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do(stream(), ptr(t), ptr(t), ptr(t), ptr(t), ptr(t), None,
                                                             32, 0, 0, 0, 2, None, 0) == -1
    assert lib.secure_infer_aicpu_gcm_encrypt_tag_do(stream(), ptr(t), ptr(t), ptr(t), ptr(t), ptr(t), 32,
                                                      0, 0, 0, 2, None, 64) == -1
    assert lib.secure_infer_aicpu_auth_gate_do(stream(), ptr(t), None, 32) == -1
