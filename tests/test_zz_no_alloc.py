"""The allocation-free decrypt/verify entry point against the regular one.

secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do is for callers that
cannot call cudaMalloc (code running inside an allocator or memory budget it
does not own, or a path that must never pay for a device allocation): it keeps
its scratch in a fixed device array instead of allocating per stream.  Its
results must equal secure_infer_aicpu_gcm_decrypt_verify_aad_do's byte for
byte, on consecutive calls that reuse the shared scratch with different keys,
sizes and outcomes.  This file sorts last so a stop-at-first-failure run has
already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes as ct
import struct

import pytest

from conftest import det_bytes
from oracle import gcm as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import _native
    return _native.lib()


def dev(data: bytes):
    return torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()


def p(t):
    return ct.c_void_p(t.data_ptr())


def at_offset(t, off: int):
    """A device copy of `t` that starts `off` bytes past a 256-byte boundary."""
    buf = torch.zeros(t.numel() + off, dtype=torch.uint8, device="cuda")
    buf[off:] = t
    return buf, ct.c_void_p(buf.data_ptr() + off)


def run(fn, stream, case, in_off=0, out_off=0):
    """One call of `fn`; in_off / out_off place the ciphertext / plaintext
    output 1..15 bytes off 16-byte alignment (the kernel's unaligned path)."""
    key, h, c, tag, aad, iv = case
    cbuf, cptr = at_offset(c, in_off)
    obuf = torch.full((len(c) + out_off,), 0xA5, dtype=torch.uint8, device="cuda")
    optr = ct.c_void_p(obuf.data_ptr() + out_off)
    st = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    aptr, alen = (p(aad), aad.numel()) if aad is not None else (None, 0)
    rc = fn(stream, cptr, p(key), p(h), p(tag), optr, p(st), c.numel(), *iv, aptr, alen)
    torch.cuda.synchronize()
    assert bool((obuf[:out_off] == 0xA5).all())          # nothing written before the output
    return rc, obuf[out_off:].cpu().numpy().tobytes(), int(st.item())


def make_case(seed: str, count: int, tamper: bool = False, aad_bytes: int = 64):
    key = det_bytes(seed + "k", 16)
    iv = [*struct.unpack(">III", det_bytes(seed + "n", 12)), 2]
    aad = det_bytes(seed + "a", aad_bytes)
    plain = det_bytes(seed + "p", count)
    h = orc.aes_block(key, bytes(16))
    c, tag = orc.gcm_encrypt_tag(plain, key, h, iv, aad)
    if tamper:
        c = c[:5] + bytes([c[5] ^ 0x20]) + c[6:]
    return (dev(key), dev(h), dev(c), dev(tag), dev(aad) if aad_bytes else None, iv), plain


def test_noalloc_matches_regular_entry_point_on_consecutive_calls(lib):
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    regular = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do
    noalloc = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do
    cases = [make_case("na1", 262144), make_case("na2", 100000 + 7), make_case("na3", 4096, tamper=True)]
    for (case, plain), expect_ok in zip(cases, (1, 1, 0)):
        rc_a, out_a, st_a = run(noalloc, stream, case)
        rc_b, out_b, st_b = run(regular, stream, case)
        assert rc_a == 0 and rc_b == 0
        assert st_a == st_b == expect_ok
        assert out_a == out_b
        assert out_a == (plain if expect_ok else bytes(len(plain)))
    # Same inputs twice in a row through the shared scratch: same answer.
    case, plain = cases[0]
    assert run(noalloc, stream, case) == (0, plain, 1)
    assert run(noalloc, stream, case) == (0, plain, 1)


@pytest.mark.parametrize("count", [16, 31, 32768 + 5])
def test_noalloc_without_aad(lib, count):
    """aad = NULL, aad_bytes = 0: GHASH over the payload alone, as the oracle
    computes it, on two calls in a row."""
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    regular = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do
    noalloc = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do
    case, plain = make_case(f"nz{count}", count, aad_bytes=0)
    want = run(regular, stream, case)
    assert want == (0, plain, 1)
    assert run(noalloc, stream, case) == want
    assert run(noalloc, stream, case) == want
    bad, _ = make_case(f"nz{count}", count, tamper=True, aad_bytes=0)
    assert run(noalloc, stream, bad) == run(regular, stream, bad) == (0, bytes(count), 0)


@pytest.mark.parametrize("in_off,out_off", [(1, 0), (0, 7), (15, 3), (8, 8)])
def test_noalloc_unaligned_buffers(lib, in_off, out_off):
    """Ciphertext and output off 16-byte alignment take the kernel's
    unaligned-record path; results equal the regular entry point's and the
    oracle's byte for byte, tampered records included."""
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    regular = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_do
    noalloc = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do
    for count, tamper in ((65536 + 9, False), (4000, True)):
        case, plain = make_case(f"nu{in_off}.{out_off}.{count}", count, tamper=tamper)
        want = (0, bytes(count) if tamper else plain, 0 if tamper else 1)
        assert run(regular, stream, case, in_off, out_off) == want
        assert run(noalloc, stream, case, in_off, out_off) == want
        assert run(noalloc, stream, case, in_off, out_off) == want


def test_noalloc_rejects_sizes_beyond_its_scratch(lib):
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    t = torch.zeros(64, dtype=torch.uint8, device="cuda")
    fn = lib.secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do
    assert fn(stream, p(t), p(t), p(t), p(t), p(t), p(t), (16 << 20) + 1, 0, 0, 0, 2, p(t), 64) == -2
    assert fn(stream, p(t), p(t), p(t), p(t), p(t), p(t), 64, 0, 0, 0, 2, p(t), 4097) == -2
    assert fn(stream, p(t), p(t), p(t), p(t), p(t), None, 64, 0, 0, 0, 2, p(t), 64) == -1
