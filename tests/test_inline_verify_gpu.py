"""GPU parity of the fused verify kernel that computes the AES keystream
itself (secure_infer_reload_records with no keystream buffer, raw records and
16-byte aligned destinations), against the host plaintext and against the
two-kernel path with a prefetched keystream.  Tampered ciphertext, tags and
AAD must come back with status 0 and a zeroed destination."""
from __future__ import annotations

import ctypes as ct

import pytest

from conftest import det_bytes

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("inline-key", 16)
SALT = det_bytes("inline-salt", 4)


@pytest.fixture(scope="module")
def nl():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield native_layerwise
    s.close()


def encrypt(nl, plain):
    """Host-encrypted records of the rows of `plain` (uint8 [n, count])."""
    lib = nl._native.lib()
    n, count = plain.shape
    stride = nl.record_bytes(count)
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tk = (ct.c_uint64 * n)()
    assert lib.secure_infer_h2d_encrypt_records(nl._ptrs(plain.data_ptr() + i * count for i in range(n)), count, n,
                                                recs.data_ptr(), stride, tk) == 0
    return recs, tk, stride


def reload(nl, drecs, stride, count, tk, dest, order, keystream):
    lib = nl._native.lib()
    n = len(order)
    status = torch.full((n,), 7, dtype=torch.int32, device="cuda")
    dsts = nl._ptrs(dest.data_ptr() + j * dest.stride(0) * dest.element_size() for j in order)
    assert lib.secure_infer_reload_records(3, drecs.data_ptr(), stride, count, n, tk, dsts, keystream,
                                           status.data_ptr(), None, nl._stream(), None) == 0
    torch.cuda.synchronize()
    return status.cpu().tolist()


# (262144, 96) is a c2 layer: one segment per warp, partials pre-scaled (the
# single pass that swaps the combine tables into shared memory).  (65536,
# 1100) gives the first launch of 1024 records several segments per warp with
# pre-scaled partials; (4 MiB + 16, 12) gives records of more than 64 segments
# (tree join by the completing warp).
@pytest.mark.parametrize("count,n", [(262144, 96), (262144 + 16, 5), (1000, 9), (16, 40), (4097, 1030),
                                     (65536, 1100), ((4 << 20) + 16, 12)])
def test_inline_keystream_reload_matches_plaintext_and_prefetched_path(nl, count, n):
    g = torch.Generator().manual_seed(count * 7 + n)
    plain = torch.randint(0, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    recs, tk, stride = encrypt(nl, plain)
    drecs = recs.cuda()
    order = torch.randperm(n + 3, generator=g)[:n].tolist()        # a random block table
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    outs = []
    for keystream in (None, ks.data_ptr()):
        dest = torch.full((n + 3, count), 0x5A, dtype=torch.uint8, device="cuda")
        assert reload(nl, drecs, stride, count, tk, dest, order, keystream) == [1] * n
        got = dest.cpu()
        assert torch.equal(got[order], plain)
        untouched = sorted(set(range(n + 3)) - set(order))
        assert got[untouched].eq(0x5A).all()
        outs.append(got)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("count", [262144 + 5, (4 << 20) + 5])
def test_inline_keystream_reload_rejects_tampering(nl, count):
    """Flip one bit of record 1's ciphertext (first block), record 3's tag,
    record 4's AAD and record 6's last payload byte: those records fail closed
    (status 0, destination zeroed), the others land.  The second size gives
    records of more than 64 segments (joined by the completing warp)."""
    n = 8
    g = torch.Generator().manual_seed(99)
    plain = torch.randint(0, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    recs, tk, stride = encrypt(nl, plain)
    aligned = (count + 31) // 32 * 32
    recs[1, 0] ^= 1
    recs[3, aligned + 7] ^= 0x80
    recs[4, aligned + 32 + 40] ^= 0x04
    recs[6, count - 1] ^= 0x10
    drecs = recs.cuda()
    order = list(range(n))
    bad = {1, 3, 4, 6}
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    for keystream in (None, ks.data_ptr()):
        dest = torch.full((n, count), 0x5A, dtype=torch.uint8, device="cuda")
        status = reload(nl, drecs, stride, count, tk, dest, order, keystream)
        assert status == [0 if i in bad else 1 for i in range(n)], keystream
        got = dest.cpu()
        for i in range(n):
            if i in bad:
                assert not got[i].any(), i
            else:
                assert torch.equal(got[i], plain[i]), i


def test_fail_closed_zeroing_is_never_overtaken_by_late_plaintext(nl):
    """Every record's tag is wrong: the warp that completes a record zeroes its
    destination after every segment's plaintext stores (each warp counts its
    segment only after a warp barrier and a device-scope fence).  Many small
    records and repeated launches give a late store many chances to land after
    the zeroing; not one destination byte may survive."""
    n, count = 1024, 4097
    g = torch.Generator().manual_seed(7)
    plain = torch.randint(1, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    recs, tk, stride = encrypt(nl, plain)
    aligned = (count + 31) // 32 * 32
    recs[:, aligned] ^= 1                      # every tag
    drecs = recs.cuda()
    order = list(range(n))
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    for rep in range(4):
        for keystream in (None, ks.data_ptr()):
            dest = torch.full((n, count), 0x5A, dtype=torch.uint8, device="cuda")
            assert reload(nl, drecs, stride, count, tk, dest, order, keystream) == [0] * n
            assert int(dest.count_nonzero().item()) == 0, (rep, keystream)


def test_layer_sm_limit_keeps_both_paths_exact(nl):
    """With each layer launch limited to a few SMs (segments sized for them),
    the fused and the two-kernel reload still land the plaintext and reject a
    tampered record; the limit is process-wide and restored afterwards."""
    lib = nl._native.lib()
    n, count = 96, 32768
    g = torch.Generator().manual_seed(11)
    plain = torch.randint(0, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    recs, tk, stride = encrypt(nl, plain)
    recs[5, count // 2] ^= 2
    drecs = recs.cuda()
    order = torch.randperm(n + 4, generator=g)[:n].tolist()
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    for sms in (7, 74):
        prev = lib.secure_infer_set_layer_sm_limit(sms)
        try:
            for keystream in (None, ks.data_ptr()):
                dest = torch.full((n + 4, count), 0x5A, dtype=torch.uint8, device="cuda")
                assert reload(nl, drecs, stride, count, tk, dest, order, keystream) == [0 if i == 5 else 1 for i in range(n)]
                got = dest.cpu()
                good = [i for i in range(n) if i != 5]
                assert torch.equal(got[[order[i] for i in good]], plain[good]), (sms, keystream)
                assert not got[order[5]].any()
        finally:
            assert lib.secure_infer_set_layer_sm_limit(prev) == sms
