"""GPU parity of the codec paths at the benchmark configs' shapes, against the
reference codec's own outputs (tests/golden/codec_shapes.json, digests of
transport_codec.encode packets and optimized_decode.decode_into blocks).

* c3_h4: Qwen2.5-7B shard shape, 4 KV heads, int8 and int4, 1% outliers at 8 sigma
* c4_h8: Llama-3-8B, 8 KV heads, int8 (layer 10) and int4 (layer 11): the two
  halves of the mixed split
* c5_h1: Llama-3-70B TP=8 shard, 1 KV head, int4, 64 blocks

Reload: the reference packets (the oracle's encode, pinned to the fixture's
digest) go through the authenticated C-ABI reload into a paged cache at the
fixture's block table; the decoded blocks must hash to the reference
decode_into output and every other block must stay zero.  Writeback: the
source blocks go through the device quantise + encrypt + tag; every record
must decrypt and verify under OpenSSL to the reference packet."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest

from conftest import codec_shape_source, codec_shapes, det_bytes, sha256
from oracle import codec_oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("shape-key", 16)
SALT = det_bytes("shape-salt", 4)
CASES = [(name, tag) for name, e in codec_shapes().items() for tag in e["cases"]]
PAIRS = [(name, bits) for name, e in codec_shapes().items() for bits in sorted({c["bits"] for c in e["cases"].values()})]


@pytest.fixture(scope="module")
def nl():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield native_layerwise
    s.close()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def reference_packets(e: dict, c: dict, src: np.ndarray) -> np.ndarray:
    packet, _, _ = codec_oracle.encode(src, e["enc_idx"], c["bits"], c["kind"], c["layer"])
    assert sha256(packet) == c["packet_sha256"]
    return packet


@pytest.mark.parametrize("name,tag", CASES)
def test_reload_at_config_shape_matches_reference_decode(nl, name, tag):
    e = codec_shapes()[name]
    c = e["cases"][tag]
    heads, bits, kind, layer = e["heads"], c["bits"], c["kind"], c["layer"]
    packets = torch.from_numpy(reference_packets(e, c, codec_shape_source(e))).pin_memory()
    b, width = packets.shape
    assert width == nl.packet_bytes(heads, bits)
    nl.register_host_range(packets, layer, kind)
    dest = torch.zeros((e["dst_blocks"], 128, heads, 128), dtype=torch.bfloat16, device="cuda")
    lib = nl._native.lib()
    srcs = nl._ptrs(packets.data_ptr() + i * width for i in range(b))
    dsts = nl._ptrs(dest.data_ptr() + i * dest.stride(0) * 2 for i in e["dst_idx"])
    codec = nl._native.Codec(bits, kind, heads, layer)
    assert lib.secure_infer_h2d_reload_layer(layer, srcs, dsts, b, width, ct.byref(codec), 0, None,
                                             nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == 0
    got = u16(dest)
    assert sha256(got[e["dst_idx"]]) == c["dest_sha256"]
    others = np.setdiff1d(np.arange(e["dst_blocks"]), e["dst_idx"])
    assert not got[others].any()


@pytest.mark.parametrize("name,bits", PAIRS)
def test_reload_kv_pair_at_config_shape(nl, name, bits):
    """K and V of a layer as one 2n-record request (SECURE_INFER_KIND_KV), the
    bench's own request shape."""
    e = codec_shapes()[name]
    src = codec_shape_source(e)
    heads = e["heads"]
    lib = nl._native.lib()
    dest = [torch.zeros((e["dst_blocks"], 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    packets, srcs, dsts, layer = [], [], [], None
    for kind in range(2):
        c = e["cases"][f"k{kind}_b{bits}"]
        layer = c["layer"]
        pk = torch.from_numpy(reference_packets(e, c, src)).pin_memory()
        nl.register_host_range(pk, layer, kind)
        packets.append(pk)
        width = pk.shape[1]
        srcs += [pk.data_ptr() + i * width for i in range(pk.shape[0])]
        dsts += [dest[kind].data_ptr() + i * dest[kind].stride(0) * 2 for i in e["dst_idx"]]
    codec = nl._native.Codec(bits, nl._native.KIND_KV, heads, layer)
    assert lib.secure_infer_h2d_reload_layer(layer, nl._ptrs(srcs), nl._ptrs(dsts), len(srcs), width,
                                             ct.byref(codec), 0, None, nl._stream()) == 0
    assert lib.secure_infer_recovery_wait_layer_authentication(layer) == 0
    for kind in range(2):
        assert sha256(u16(dest[kind])[e["dst_idx"]]) == e["cases"][f"k{kind}_b{bits}"]["dest_sha256"], kind


@pytest.mark.parametrize("name,bits", PAIRS)
def test_writeback_at_config_shape_gives_reference_packets(nl, name, bits):
    """Device gather + quantise + encrypt + tag of the fixture's source blocks
    (K and V in one request, from a paged cache): each record verifies under
    OpenSSL and decrypts to the reference's packet."""
    from oracle import gcm as orc
    e = codec_shapes()[name]
    heads = e["heads"]
    src = codec_shape_source(e)
    lib = nl._native.lib()
    # The source blocks sit in a device paged cache in reverse order, so the
    # gather follows a non-trivial block table.
    nb = e["blocks"]
    cache = torch.from_numpy(src[::-1].copy().view(np.int16)).view(torch.bfloat16).cuda()
    bb = 128 * heads * 128 * 2
    layer = e["cases"][f"k0_b{bits}"]["layer"]
    count = nl.packet_bytes(heads, bits)
    stride = nl.record_bytes(count)
    aligned = orc.record_aligned_bytes(count)
    n1 = len(e["enc_idx"])
    n = 2 * n1
    srcs = nl._ptrs(cache.data_ptr() + (nb - 1 - i) * bb for _ in range(2) for i in e["enc_idx"])
    records = torch.zeros((n, stride), dtype=torch.uint8, device="cuda")
    tickets = (ct.c_uint64 * n)()
    codec = nl._native.Codec(bits, nl._native.KIND_KV, heads, layer)
    assert lib.secure_infer_writeback_records(srcs, None, n, ct.byref(codec), records.data_ptr(), stride, tickets,
                                              nl._stream()) == 0
    torch.cuda.synchronize()
    recs = records.cpu().numpy()
    for kind in range(2):
        c = e["cases"][f"k{kind}_b{bits}"]
        want = reference_packets(e, c, src)
        rows = []
        for j in range(n1):
            rec = recs[kind * n1 + j].tobytes()
            aad = rec[aligned + 32:aligned + 96]
            iv = orc.derive_transfer_iv(SALT, tickets[kind * n1 + j])
            plain, ok = orc.host_decrypt_verify(KEY, iv, aad, rec[:count], rec[aligned:aligned + 16])
            assert ok == 1, (kind, j)
            rows.append(np.frombuffer(plain, np.uint8))
        got = np.stack(rows)
        if sha256(got) != c["packet_sha256"]:
            bad = [j for j in range(n1) if not np.array_equal(got[j], want[j])]
            pytest.fail(f"kind {kind}: packets of rows {bad[:8]} differ from the reference's")
