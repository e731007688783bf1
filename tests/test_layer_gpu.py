"""GPU parity of the per-layer reload and writeback paths through the C ABI.

Reload: host records -> staged H2D -> keystream -> fused verify/XOR/(dequant)
/scatter into a paged cache via a random block table; compared with the raw
host blocks (KV_CODEC=none) or with the reference codec's own decode_into
output (golden fixtures, bit-exact).  Writeback: device blocks -> quantise +
encrypt + tag -> host verify; packets compared with the oracle encode."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest

from conftest import det_bytes, load_codec
from oracle import codec_oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("layer-key", 16)
SALT = det_bytes("layer-salt", 4)


@pytest.fixture(scope="module")
def nl():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield native_layerwise
    s.close()


def bf16_random(shape, seed, outliers=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g)
    if outliers:
        m = torch.rand(shape, generator=g) < 0.01
        x = torch.where(m, 8.0 * torch.sign(torch.randn(shape, generator=g)), x)
    return x.to(torch.bfloat16)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("heads,blocks,n", [(8, 6, 4), (1, 3, 3), (2, 48, 48)])
def test_reload_layer_raw(nl, heads, blocks, n):
    layer = 3
    host = [bf16_random((blocks, 128, heads, 128), 10 + k).pin_memory() for k in range(2)]
    for k in range(2):
        nl.register_host_range(host[k], layer, k)
    cache = [torch.zeros((blocks + 5, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    perm = torch.randperm(blocks + 5, generator=torch.Generator().manual_seed(1))[:n]
    src_ids = torch.randperm(blocks, generator=torch.Generator().manual_seed(2))[:n]
    mapping = torch.stack((src_ids, perm), 1)
    t = nl.NativeTransfer("none", layers=32)
    t.layer = layer
    t.single_layer_kv_transfer((host, mapping), cache)
    t.wait_for_layer_load(layer)
    torch.cuda.synchronize()
    for k in range(2):
        got = cache[k].cpu()
        assert torch.equal(got[perm], host[k][src_ids])
        mask = torch.ones(blocks + 5, dtype=torch.bool)
        mask[perm] = False
        assert not got[mask].view(torch.int16).any()


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("bits", [8, 4])
def test_reload_codec_matches_reference_decode(nl, heads, kind, bits):
    """Packets made by the reference encode, authenticated + decoded on the GPU,
    must equal the reference decode_into output bit for bit."""
    g = load_codec(heads)
    tag = f"k{kind}_b{bits}"
    packets = torch.from_numpy(g[f"packet_{tag}"]).pin_memory()     # [b, width]
    b, width = packets.shape
    assert width == nl.packet_bytes(heads, bits)
    layer = 1 if bits == 8 else 20
    nl.register_host_range(packets, layer, kind)
    dest = torch.zeros((6, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    dst_idx = [int(i) for i in g["dst_idx"]]
    lib = nl._native.lib()
    srcs = nl._ptrs(packets.data_ptr() + i * width for i in range(b))
    dsts = nl._ptrs(dest.data_ptr() + i * dest.stride(0) * 2 for i in dst_idx)
    codec = nl._native.Codec(bits, kind, heads, layer)
    assert lib.secure_infer_h2d_reload_layer(layer, srcs, dsts, b, width, ct.byref(codec), 0, None,
                                             nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == 0
    got = u16(dest)
    assert np.array_equal(got[dst_idx], g[f"dest_{tag}"])
    others = np.setdiff1d(np.arange(6), dst_idx)
    assert not got[others].any()


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("bits", [8, 4])
def test_reload_codec_kv_pair_matches_reference_decode(nl, heads, bits):
    """K and V packets of one layer reloaded as one 2n-record request
    (SECURE_INFER_KIND_KV), both decoded bit-exact like decode_into."""
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
    assert lib.secure_infer_h2d_reload_layer(layer, nl._ptrs(srcs), nl._ptrs(dsts), len(srcs), width,
                                             ct.byref(codec), 0, None, nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == 0
    for kind in range(2):
        got = u16(dest[kind])
        assert np.array_equal(got[dst_idx], g[f"dest_k{kind}_b{bits}"]), kind
    # An odd record count cannot be split into K and V halves.
    assert lib.secure_infer_h2d_reload_layer(layer, nl._ptrs(srcs), nl._ptrs(dsts), len(srcs) - 1, width,
                                             ct.byref(codec), 0, None, nl._stream()) == -1


@pytest.mark.parametrize("mode", ["int8", "int4", "mixed"])
def test_native_transfer_codec_layers(nl, mode):
    """NativeTransfer over several layers with the per-layer bit split."""
    heads, blocks, layers = 2, 5, 4
    src = bf16_random((blocks, 128, heads, 128), 77, outliers=True)
    dest = [torch.zeros((blocks + 2, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    mapping = torch.stack((torch.arange(blocks), torch.arange(blocks).flip(0) + 2), 1)
    t = nl.NativeTransfer(mode, layers=layers)
    for layer in range(layers):
        bits = nl.layer_bits(mode, layer, layers)
        host = []
        for kind in range(2):
            pk, qb, sb = codec_oracle.encode(u16(src), np.arange(blocks), bits, kind, layer)
            host.append(torch.from_numpy(pk).pin_memory())
            nl.register_host_range(host[-1], layer, kind)
        t.single_layer_kv_transfer((host, mapping), dest)
        t.wait_for_layer_load(layer)
        for kind in range(2):
            ref = np.zeros((blocks + 2, 128, heads, 128), np.uint16)
            pk = host[kind].numpy()
            qb = 128 * heads * 128 * bits // 8
            sb = 128 * heads * 128 // 64 * 4
            codec_oracle.decode_into(pk, ref, mapping[:, 1].numpy(), bits, kind, qb, sb)
            assert np.array_equal(u16(dest[kind]), ref), (layer, kind)


def test_tamper_then_strict_retry(nl):
    heads, blocks = 2, 4
    layer = 7
    host = [bf16_random((blocks, 128, heads, 128), 30 + k).pin_memory() for k in range(2)]
    for k in range(2):
        nl.register_host_range(host[k], layer, k)
    cache = [torch.zeros((blocks, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    mapping = torch.stack((torch.arange(blocks), torch.arange(blocks)), 1)
    lib = nl._native.lib()
    before = nl.auth_stats()
    lib.secure_infer_arm_tamper(1, 3, 0)          # 3rd record: ciphertext byte flipped
    t = nl.NativeTransfer("none", layers=32)
    t.layer = layer
    t.single_layer_kv_transfer((host, mapping), cache)
    t.wait_for_layer_load(layer)                  # retried once with a fresh ticket -> ok
    after = nl.auth_stats()
    assert after["rejected"] - before["rejected"] == 1
    assert after["retried"] - before["retried"] == 1
    for k in range(2):
        assert torch.equal(cache[k].cpu(), host[k])


def test_tamper_precencrypted_is_fatal_and_zeroed(nl):
    """Pre-encrypted records have no trusted plaintext to retry from: the
    tampered record's destination is zeroed and the wait reports -1."""
    heads, n, layer = 1, 3, 9
    host = bf16_random((n, 128, heads, 128), 55).pin_memory()
    nl.register_host_range(host, layer, 0)
    count = host[0].numel() * 2
    lib = nl._native.lib()
    stride = nl.record_bytes(count)
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tickets = (ct.c_uint64 * n)()
    srcs = nl._ptrs(host.data_ptr() + i * count for i in range(n))
    assert lib.secure_infer_h2d_encrypt_records(srcs, count, n, recs.data_ptr(), stride, tickets) == 0
    aligned = (count + 31) // 32 * 32
    recs[1, aligned + 3] ^= 0x40                  # flip a tag byte
    dest = torch.full((n, 128, heads, 128), 3.0, dtype=torch.bfloat16, device="cuda")
    dsts = nl._ptrs(dest.data_ptr() + i * count for i in range(n))
    rsrc = nl._ptrs([recs.data_ptr()])
    assert lib.secure_infer_h2d_reload_layer(layer, rsrc, dsts, n, count, None, 1, tickets, nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == -1
    got = dest.cpu()
    assert torch.equal(got[0], host[0]) and torch.equal(got[2], host[2])
    assert not got[1].view(torch.int16).any()
    # Replaying the same tickets is rejected before any device work.
    assert lib.secure_infer_h2d_reload_layer(layer, rsrc, dsts, n, count, None, 1, tickets, nl._stream()) == -1


@pytest.mark.parametrize("bits", [8, 4])
def test_codec_tamper_fails_closed(nl, bits):
    """A K+V codec reload where one record's quantised bytes, one record's
    scale array and one record's tag were altered: exactly those records get
    status 0 and their whole bf16 destination block zeroed, the rest decode."""
    from oracle import gcm as orc
    heads, layer = 2, 13
    lib = nl._native.lib()
    cache = bf16_random((8, 128, heads, 128), 700 + bits).cuda()
    ids = [5, 1, 6, 2, 7, 0]
    n = len(ids)
    bb = 128 * heads * 128 * 2
    count = nl.packet_bytes(heads, bits)
    stride = nl.record_bytes(count)
    aligned = orc.record_aligned_bytes(count)
    qb = 128 * heads * 128 * bits // 8
    records = torch.zeros((n, stride), dtype=torch.uint8, device="cuda")
    tickets = (ct.c_uint64 * n)()
    codec = nl._native.Codec(bits, nl._native.KIND_KV, heads, layer)
    assert lib.secure_infer_writeback_records(nl._ptrs(cache.data_ptr() + i * bb for i in ids), None, n,
                                              ct.byref(codec), records.data_ptr(), stride, tickets,
                                              nl._stream()) == 0
    torch.cuda.synchronize()
    records[1, qb // 2] ^= 0x10          # K record: quantised byte
    records[3, qb + 8] ^= 0x01           # V record: scale array
    records[4, aligned + 5] ^= 0x80      # V record: tag
    dest = torch.full((n, 128, heads, 128), 2.0, dtype=torch.bfloat16, device="cuda")
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    status = torch.full((n,), 7, dtype=torch.int32, device="cuda")
    assert lib.secure_infer_reload_records(layer, records.data_ptr(), stride, count, n, tickets,
                                           nl._ptrs(dest.data_ptr() + i * bb for i in range(n)), ks.data_ptr(),
                                           status.data_ptr(), ct.byref(codec), nl._stream(), None) == 0
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [1, 0, 1, 0, 0, 1]
    got = u16(dest)
    src = u16(cache)
    for i in range(n):
        if i in (1, 3, 4):
            assert not got[i].any(), i
        else:
            kind = 0 if i < n // 2 else 1
            pk, q_b, s_b = codec_oracle.encode(src, [ids[i]], bits, kind, layer)
            exp = np.zeros((1, 128, heads, 128), np.uint16)
            codec_oracle.decode_into(pk, exp, [0], bits, kind, q_b, s_b)
            assert np.array_equal(got[i], exp[0]), i


def test_reload_records_device_resident(nl):
    heads, n, layer = 4, 8, 2
    host = bf16_random((n, 128, heads, 128), 66).pin_memory()
    nl.register_host_range(host, layer, 1)
    count = host[0].numel() * 2
    lib = nl._native.lib()
    stride = nl.record_bytes(count)
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tickets = (ct.c_uint64 * n)()
    srcs = nl._ptrs(host.data_ptr() + i * count for i in range(n))
    assert lib.secure_infer_h2d_encrypt_records(srcs, count, n, recs.data_ptr(), stride, tickets) == 0
    drecs = recs.cuda()
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    dest = torch.zeros((n, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    order = list(reversed(range(n)))
    dsts = nl._ptrs(dest.data_ptr() + i * count for i in order)
    for keystream in (ks.data_ptr(), None):       # prefetched keystream / AES inline
        dest.zero_()
        status.zero_()
        assert lib.secure_infer_reload_records(layer, drecs.data_ptr(), stride, count, n, tickets, dsts, keystream,
                                               status.data_ptr(), None, nl._stream(), None) == 0
        torch.cuda.synchronize()
        assert status.cpu().tolist() == [1] * n
        assert torch.equal(dest.cpu()[order], host)


@pytest.mark.parametrize("count,n,dst_offset", [(1000, 7, 4), (48, 1500, 0), (16, 3, 2), (4097, 33, 0),
                                                 (1 << 20, 1, 0), (300000, 2, 0), (262144, 3, 0)])
def test_reload_records_odd_sizes_and_chunks(nl, count, n, dst_offset):
    """Device-resident reload of raw records whose size is not a multiple of
    16, into unaligned destinations, and more records than one launch holds
    (1024): every byte lands, nothing past `count` is written."""
    lib = nl._native.lib()
    stride = nl.record_bytes(count)
    g = torch.Generator().manual_seed(count + n)
    plain = torch.randint(0, 256, (n, count), dtype=torch.uint8, generator=g).pin_memory()
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tk = (ct.c_uint64 * n)()
    assert lib.secure_infer_h2d_encrypt_records(nl._ptrs(plain.data_ptr() + i * count for i in range(n)), count, n,
                                                recs.data_ptr(), stride, tk) == 0
    drecs = recs.cuda()
    pitch = count + 64
    dest = torch.full((n, pitch), 0xA5, dtype=torch.uint8, device="cuda")
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    for keystream in (ks.data_ptr(), None):
        dest.fill_(0xA5)
        status.zero_()
        assert lib.secure_infer_reload_records(1, drecs.data_ptr(), stride, count, n, tk,
                                               nl._ptrs(dest.data_ptr() + i * pitch + dst_offset for i in range(n)),
                                               keystream, status.data_ptr(), None, nl._stream(), None) == 0
        torch.cuda.synchronize()
        got = dest.cpu()
        assert status.cpu().eq(1).all()
        assert torch.equal(got[:, dst_offset:dst_offset + count], plain)
        assert got[:, :dst_offset].eq(0xA5).all() and got[:, dst_offset + count:].eq(0xA5).all()


def test_reload_records_shared_keystream_across_streams(nl):
    """Consecutive reloads that share one keystream buffer, with the keystream
    on the session's producer stream: each layer's output must be its own."""
    heads, n, layers = 2, 6, 4
    lib = nl._native.lib()
    count = 128 * heads * 128 * 2
    stride = nl.record_bytes(count)
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    side = torch.cuda.Stream()
    hosts, drecs, tks, dests, status = [], [], [], [], torch.zeros((layers, n), dtype=torch.int32, device="cuda")
    for layer in range(layers):
        host = bf16_random((n, 128, heads, 128), 300 + layer).pin_memory()
        nl.register_host_range(host, 40 + layer, 0)
        recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
        tk = (ct.c_uint64 * n)()
        srcs = nl._ptrs(host.data_ptr() + i * count for i in range(n))
        assert lib.secure_infer_h2d_encrypt_records(srcs, count, n, recs.data_ptr(), stride, tk) == 0
        hosts.append(host)
        drecs.append(recs.cuda())
        tks.append(tk)
        dests.append(torch.zeros((n, 128, heads, 128), dtype=torch.bfloat16, device="cuda"))
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        for layer in range(layers):
            dsts = nl._ptrs(dests[layer].data_ptr() + i * count for i in range(n))
            assert lib.secure_infer_reload_records(40 + layer, drecs[layer].data_ptr(), stride, count, n, tks[layer],
                                                   dsts, ks.data_ptr(), status[layer].data_ptr(), None,
                                                   nl._stream(side), None) == 0
    torch.cuda.synchronize()
    assert status.cpu().eq(1).all()
    for layer in range(layers):
        assert torch.equal(dests[layer].cpu(), hosts[layer]), layer


def test_kernel_profile_counts_reload_launches(nl):
    """secure_infer_kernel_profile_*: one device-resident reload of a layer is
    one keystream launch and one verify launch, each with a device time."""
    heads, n = 2, 4
    lib = nl._native.lib()
    count = 128 * heads * 128 * 2
    stride = nl.record_bytes(count)
    host = bf16_random((n, 128, heads, 128), 901).pin_memory()
    recs = torch.zeros((n, stride), dtype=torch.uint8).pin_memory()
    tk = (ct.c_uint64 * n)()
    assert lib.secure_infer_h2d_encrypt_records(nl._ptrs(host.data_ptr() + i * count for i in range(n)), count, n,
                                                recs.data_ptr(), stride, tk) == 0
    drecs = recs.cuda()
    dest = torch.zeros((n, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    kinds = 16
    us, cnt = (ct.c_double * kinds)(), (ct.c_uint64 * kinds)()
    torch.cuda.synchronize()
    lib.secure_infer_kernel_profile_collect(us, cnt, kinds)           # drop anything recorded earlier
    assert lib.secure_infer_kernel_profile_enable(1) == 0
    try:
        s = nl._stream()
        assert lib.secure_infer_reload_records(3, drecs.data_ptr(), stride, count, n, tk,
                                               nl._ptrs(dest.data_ptr() + i * count for i in range(n)),
                                               ks.data_ptr(), status.data_ptr(), None, s, s) == 0
        torch.cuda.synchronize()
        assert lib.secure_infer_kernel_profile_collect(us, cnt, kinds) == 0
    finally:
        lib.secure_infer_kernel_profile_enable(0)
    got = {lib.secure_infer_kernel_name(k).decode(): (cnt[k], us[k]) for k in range(kinds)
           if lib.secure_infer_kernel_name(k) is not None and cnt[k]}
    assert set(got) == {"gcm_layer_ctr_kernel", "gcm_layer_verify_kernel"}
    assert all(c == 1 and t > 0 for c, t in got.values())
    assert status.cpu().tolist() == [1] * n and torch.equal(dest.cpu(), host)


def test_group_bracket_and_job_auth(nl):
    heads, blocks, layer = 1, 5, 11
    host = bf16_random((blocks, 128, heads, 128), 88).pin_memory()
    nl.register_host_range(host, layer, 0)
    cache = torch.zeros((blocks, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    lib = nl._native.lib()
    count = host[0].numel() * 2
    lib.secure_infer_recovery_set_job_id(1234)
    assert lib.secure_infer_h2d_layer_group_begin(blocks) == 0
    for i in range(blocks):
        assert lib.secure_infer_h2d_submit(cache.data_ptr() + i * count, count, host.data_ptr() + i * count, count,
                                           nl._stream()) == 0
    assert lib.secure_infer_h2d_layer_group_end() == 0
    assert lib.secure_infer_recovery_wait_job_authentication(1234) == 1
    assert lib.secure_infer_recovery_wait_job_authentication(1234) == -1
    lib.secure_infer_recovery_set_job_id(0)
    assert torch.equal(cache.cpu(), host)


@pytest.mark.parametrize("bits", [0, 8, 4])
@pytest.mark.parametrize("kind", [0, 1])
def test_writeback_roundtrip(nl, bits, kind):
    heads, blocks, layer = 2, 5, 6
    cache = bf16_random((blocks + 3, 128, heads, 128), 99 + bits + kind, outliers=True).cuda()
    block_ids = [6, 1, 4, 0, 7]
    if bits:
        width = nl.packet_bytes(heads, bits)
        host = torch.zeros((blocks + 1, width), dtype=torch.uint8).pin_memory()
    else:
        host = torch.zeros((blocks + 1, 128, heads, 128), dtype=torch.bfloat16).pin_memory()
    nl.register_host_range(host, layer, kind)
    host_ids = [5, 0, 2, 1, 3]
    nl.store_layer(cache, block_ids, host, host_ids, kind=kind, layer=layer, bits=bits)
    nl.wait_stores()
    src = u16(cache)[block_ids]
    if bits:
        ref, _, _ = codec_oracle.encode(u16(cache), block_ids, bits, kind, layer)
        assert np.array_equal(host.numpy()[host_ids], ref)
        # Round trip back through the authenticated reload path.
        dest = [torch.zeros((blocks, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        t = nl.NativeTransfer("int8" if bits == 8 else "int4", layers=32)
        t.layer = layer
        mapping = torch.stack((torch.tensor(host_ids), torch.arange(blocks)), 1)
        pair = [host, host]
        t.single_layer_kv_transfer((pair, mapping), dest)
        t.wait_for_layer_load(layer)
        exp = np.zeros((blocks, 128, heads, 128), np.uint16)
        qb = 128 * heads * 128 * bits // 8
        sb = 128 * heads * 128 // 64 * 4
        codec_oracle.decode_into(ref, exp, np.arange(blocks), bits, kind, qb, sb)
        assert np.array_equal(u16(dest[kind]), exp)
    else:
        assert np.array_equal(u16(host)[host_ids], src)


@pytest.mark.parametrize("bits,kind", [(0, 0), (8, 0), (8, 1), (4, 0), (4, 1), (8, 2), (4, 2)])
def test_writeback_records_device_roundtrip(nl, bits, kind):
    """Device writeback (quantise + keystream + fused encrypt/tag) of a shuffled
    set of paged-cache blocks: every record must equal the oracle's OpenSSL
    view (C, tag and AAD decrypt-verify to the oracle packet or the raw block),
    then reload through reload_records back into the paged cache."""
    from oracle import gcm as orc
    heads, layer = 2, 9
    lib = nl._native.lib()
    cache = bf16_random((12, 128, heads, 128), 500 + 10 * bits + kind, outliers=True).cuda()
    ids = [7, 2, 9, 0, 11, 4] if kind == 2 else [7, 2, 9, 0, 5]
    n = len(ids)
    kinds = [0] * (n // 2) + [1] * (n - n // 2) if kind == 2 else [kind] * n
    bb = 128 * heads * 128 * 2
    count = nl.packet_bytes(heads, bits) if bits else bb
    stride = nl.record_bytes(count)
    aligned = orc.record_aligned_bytes(count)
    records = torch.zeros((n, stride), dtype=torch.uint8, device="cuda")
    tickets = (ct.c_uint64 * n)()
    srcs = nl._ptrs(cache.data_ptr() + i * bb for i in ids)
    codec = nl._native.Codec(bits, kind, heads, layer)
    assert lib.secure_infer_writeback_records(srcs, None, n, ct.byref(codec), records.data_ptr(), stride, tickets,
                                              nl._stream()) == 0
    torch.cuda.synchronize()
    recs = records.cpu().numpy()
    src = u16(cache)
    for i in range(n):
        rec = recs[i].tobytes()
        if bits:
            want, _, _ = codec_oracle.encode(src, [ids[i]], bits, kinds[i], layer)
            want = want[0].tobytes()
        else:
            want = src[ids[i]].tobytes()
        aad = rec[aligned + 32:aligned + 96]
        assert aad[:4] == b"SFAD" and aad[5] == 2           # direction D2H
        assert int.from_bytes(aad[36:44], "big") == tickets[i]
        assert rec[count:aligned] == bytes(aligned - count) and rec[aligned + 16:aligned + 32] == bytes(16)
        iv = orc.derive_transfer_iv(SALT, tickets[i])
        plain, ok = orc.host_decrypt_verify(KEY, iv, aad, rec[:count], rec[aligned:aligned + 16])
        assert ok == 1 and plain == want, i
        # The oracle's own encryption of the same plaintext gives the same record bytes.
        assert orc.host_encrypt_record(KEY, iv, aad, want)[:aligned + 16] == rec[:aligned + 16], i
    # Back through the authenticated reload path.
    dest = torch.zeros((n, 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    ks = torch.empty(n * ((count + 15) // 16 * 16 + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    dsts = nl._ptrs(dest.data_ptr() + i * bb for i in range(n))
    assert lib.secure_infer_reload_records(layer, records.data_ptr(), stride, count, n, tickets, dsts, ks.data_ptr(),
                                           status.data_ptr(), ct.byref(codec) if bits else None, nl._stream(),
                                           None) == 0
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [1] * n
    got = u16(dest)
    for i in range(n):
        if bits:
            pk, qb, sb = codec_oracle.encode(src, [ids[i]], bits, kinds[i], layer)
            exp = np.zeros((1, 128, heads, 128), np.uint16)
            codec_oracle.decode_into(pk, exp, [0], bits, kinds[i], qb, sb)
            assert np.array_equal(got[i], exp[0]), i
        else:
            assert np.array_equal(got[i], src[ids[i]]), i


def test_writeback_records_more_than_one_launch(nl):
    """1030 raw blocks (more than the 1024 records a launch holds) written back
    on the device and reloaded: every block round-trips."""
    heads, n, layer = 1, 1030, 14
    lib = nl._native.lib()
    bb = 128 * heads * 128 * 2
    cache = bf16_random((n, 128, heads, 128), 4242).cuda()
    stride = nl.record_bytes(bb)
    records = torch.zeros((n, stride), dtype=torch.uint8, device="cuda")
    tickets = (ct.c_uint64 * n)()
    codec = nl._native.Codec(0, 0, heads, layer)
    order = list(reversed(range(n)))
    assert lib.secure_infer_writeback_records(nl._ptrs(cache.data_ptr() + i * bb for i in order), None, n,
                                              ct.byref(codec), records.data_ptr(), stride, tickets,
                                              nl._stream()) == 0
    dest = torch.zeros_like(cache)
    ks = torch.empty(n * (bb + 16), dtype=torch.uint8, device="cuda")
    status = torch.zeros(n, dtype=torch.int32, device="cuda")
    assert lib.secure_infer_reload_records(layer, records.data_ptr(), stride, bb, n, tickets,
                                           nl._ptrs(dest.data_ptr() + i * bb for i in range(n)), ks.data_ptr(),
                                           status.data_ptr(), None, nl._stream(), None) == 0
    torch.cuda.synchronize()
    assert status.cpu().eq(1).all()
    assert torch.equal(dest.cpu(), cache.cpu()[order])


def test_writeback_tamper_withheld(nl):
    heads, layer = 1, 12
    cache = bf16_random((3, 128, heads, 128), 5).cuda()
    host = torch.zeros((3, 128, heads, 128), dtype=torch.bfloat16).pin_memory()
    nl.register_host_range(host, layer, 0)
    lib = nl._native.lib()
    lib.secure_infer_arm_tamper(2, 2, 0)
    nl.store_layer(cache, [0, 1, 2], host, [0, 1, 2], kind=0, layer=layer, bits=0)
    with pytest.raises(RuntimeError, match="withheld"):
        nl.wait_stores()
    got = host
    assert torch.equal(got[0], cache[0].cpu()) and torch.equal(got[2], cache[2].cpu())
    assert not got[1].view(torch.int16).any()


def test_d2h_bracket_api(nl):
    heads, layer = 1, 13
    cache = bf16_random((4, 128, heads, 128), 6).cuda()
    host = torch.zeros((4, 128, heads, 128), dtype=torch.bfloat16).pin_memory()
    nl.register_host_range(host, layer, 1)
    lib = nl._native.lib()
    count = cache[0].numel() * 2
    assert lib.secure_infer_d2h_batch_begin(1) == 0
    assert lib.secure_infer_d2h_group_begin(4) == 0
    for i in range(4):
        assert lib.secure_infer_d2h_submit(host.data_ptr() + i * count, cache.data_ptr() + (3 - i) * count, count,
                                           nl._stream()) == 0
    assert lib.secure_infer_d2h_group_end() == 0
    assert lib.secure_infer_d2h_batch_device_barrier() == 0
    assert lib.secure_infer_d2h_batch_end() == 0
    assert torch.equal(host, cache.cpu().flip(0))
