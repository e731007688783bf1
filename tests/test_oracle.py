"""Pin the CPU oracle against the golden fixtures (no GPU)."""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN, codec_shape_source, codec_shapes, det_bytes, load_codec, sha256
from oracle import codec_oracle, gcm


def test_aes_fips197_appendix_c1_shape(gcm_kat):
    # H = E_K(0^128) from the fixture (cryptography AES-ECB) must match the oracle.
    for case in gcm_kat:
        assert gcm.aes_block(bytes.fromhex(case["key"]), bytes(16)).hex() == case["h"]


@pytest.mark.parametrize("index", range(4))
def test_gcm_encrypt_tag_matches_kat(gcm_kat, index):
    case = gcm_kat[index]
    key, h = bytes.fromhex(case["key"]), bytes.fromhex(case["h"])
    aad = bytes.fromhex(case["aad"])
    plain = det_bytes(case["plain_seed"], case["count"])
    c, tag = gcm.gcm_encrypt_tag(plain, key, h, case["iv_words"], aad)
    assert tag.hex() == case["tag"]
    assert hashlib.sha256(c).hexdigest() == case["cipher_sha256"]
    if "cipher" in case:
        assert c.hex() == case["cipher"]
    _, tag0 = gcm.gcm_encrypt_tag(plain, key, h, case["iv_words"], None)
    assert tag0.hex() == case["tag_noaad"]


@pytest.mark.parametrize("index", range(4))
def test_gcm_decrypt_paths_and_tamper(gcm_kat, index):
    case = gcm_kat[index]
    key, h = bytes.fromhex(case["key"]), bytes.fromhex(case["h"])
    aad = bytes.fromhex(case["aad"])
    plain = det_bytes(case["plain_seed"], case["count"])
    c, tag = gcm.gcm_encrypt_tag(plain, key, h, case["iv_words"], aad)
    out, st = gcm.gcm_decrypt_verify(c, key, h, tag, case["iv_words"], aad)
    assert st == 1 and out == plain
    ks = gcm.keystream(key, len(c), case["iv_words"])
    out, st = gcm.gcm_verify_xor(c, key, h, tag, ks, case["iv_words"], aad)
    assert st == 1 and out == plain
    assert gcm.gcm_verify_only(c, key, h, tag, case["iv_words"], aad) == 1
    # Flip one ciphertext bit / one tag bit / one AAD bit: status 0, zeroed output.
    bad_c = bytes([c[0] ^ 1]) + c[1:]
    out, st = gcm.gcm_decrypt_verify(bad_c, key, h, tag, case["iv_words"], aad)
    assert st == 0 and out == bytes(len(c))
    bad_tag = tag[:15] + bytes([tag[15] ^ 0x80])
    out, st = gcm.gcm_verify_xor(c, key, h, bad_tag, ks, case["iv_words"], aad)
    assert st == 0 and out == bytes(len(c))
    bad_aad = bytes([aad[0] ^ 4]) + aad[1:]
    assert gcm.gcm_verify_only(c, key, h, tag, case["iv_words"], bad_aad) == 0


def test_ctr_and_ghash_flags(gcm_kat):
    case = gcm_kat[2]
    key, h = bytes.fromhex(case["key"]), bytes.fromhex(case["h"])
    aad = bytes.fromhex(case["aad"])
    plain = det_bytes(case["plain_seed"], case["count"])
    c = gcm.aes_ctr(plain, key, case["iv_words"])
    assert c.hex() == case["cipher"]
    words = list(case["iv_words"])
    words[3] = 1
    mask = gcm.keystream(key, 16, words)
    ks = gcm.keystream(key, len(c), case["iv_words"])
    tag = bytes.fromhex(case["tag"])
    out, plain_out, st = gcm.ghash_flags(c, h, aad, mask, tag, ks, 1 | 2 | 4)
    assert out == tag and st == 1 and plain_out == plain
    out, plain_out, st = gcm.ghash_flags(c, h, aad, None, None, None, 0)
    assert bytes(a ^ b for a, b in zip(out, mask)) == tag and st == 1


def test_record_layout_matches_golden(golden_records):
    key = bytes.fromhex(golden_records["key"])
    salt = bytes.fromhex(golden_records["salt"])
    for row in golden_records["rows"]:
        iv = gcm.derive_transfer_iv(salt, row["ticket"])
        assert iv.hex() == row["iv"]
        aad = gcm.build_gcm_aad(1, row["kind"], row["layer"], row["block"], 0, row["count"], row["ticket"])
        assert aad.hex() == row["aad"]
        plain = det_bytes(row["plain_seed"], row["count"])
        rec = gcm.host_encrypt_record(key, iv, aad, plain)
        assert len(rec) == row["record_len"]
        assert hashlib.sha256(rec).hexdigest() == row["record_sha256"]
        aligned = gcm.record_aligned_bytes(row["count"])
        out, ok = gcm.host_decrypt_verify(key, iv, aad, rec[:row["count"]], rec[aligned:aligned + 16])
        assert ok == 1 and out == plain
        out, ok = gcm.host_decrypt_verify(key, iv, aad, bytes([rec[0] ^ 1]) + rec[1:row["count"]],
                                          rec[aligned:aligned + 16])
        assert ok == 0 and out == bytes(row["count"])


def test_host_batch_threads_roundtrip(golden_records):
    key = np.frombuffer(bytes.fromhex(golden_records["key"]), np.uint8).copy()
    count, n = 4096, 9
    stride = gcm.record_bytes(count)
    aligned = gcm.record_aligned_bytes(count)
    records = np.zeros((n, stride), np.uint8)
    ivs = np.zeros((n, 16), np.uint8)
    plains = [np.frombuffer(det_bytes(f"b{i}", count), np.uint8).copy() for i in range(n)]
    for i in range(n):
        ivs[i] = np.frombuffer(gcm.derive_transfer_iv(b"salt", i + 1), np.uint8)
        records[i, aligned + 32:] = np.frombuffer(gcm.build_gcm_aad(1, 0, 0, i, 0, count, i + 1), np.uint8)
    st = np.zeros(n, np.uint32)
    gcm.host_batch(key, ivs, records, count, plains, st, 4, encrypt=True)
    assert st.all()
    outs = [np.zeros(count, np.uint8) for _ in range(n)]
    records[3, 5] ^= 1
    gcm.host_batch(key, ivs, records, count, outs, st, 3, encrypt=False)
    assert list(st) == [1, 1, 1, 0, 1, 1, 1, 1, 1]
    for i in range(n):
        assert (outs[i] == (0 if i == 3 else plains[i])).all()


def test_layer_bits_matches_reference():
    bits = json.loads((GOLDEN / "layer_bits.json").read_text())
    for mode, expected in bits.items():
        got = [codec_oracle.layer_bits(mode, layer, layers) for layers in (28, 32, 40, 80)
               for layer in range(layers)]
        assert got == expected


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("bits", [8, 4])
def test_codec_oracle_bit_exact_vs_reference(heads, kind, bits):
    g = load_codec(heads)
    tag = f"k{kind}_b{bits}"
    packet, qb, sb = codec_oracle.encode(g["source"], g["enc_idx"], bits, kind, layer=5)
    assert qb == int(g[f"qb_{tag}"]) and sb == int(g[f"sb_{tag}"])
    assert packet.shape == g[f"packet_{tag}"].shape
    assert np.array_equal(packet, g[f"packet_{tag}"])
    dest = np.zeros((6, 128, heads, 128), np.uint16)
    codec_oracle.decode_into(g[f"packet_{tag}"], dest, g["dst_idx"], bits, kind, qb, sb)
    assert np.array_equal(dest[g["dst_idx"]], g[f"dest_{tag}"])
    others = np.setdiff1d(np.arange(6), g["dst_idx"])
    assert not dest[others].any()


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("bits", [8, 4])
def test_codec_torch_encode_bit_exact_vs_reference(heads, kind, bits):
    """The torch CPU restatement (the CPU baseline's encode) gives the
    reference's own packets."""
    pytest.importorskip("torch")
    g = load_codec(heads)
    packet, qb, sb = codec_oracle.encode_torch(g["source"], g["enc_idx"], bits, kind, layer=5)
    assert np.array_equal(packet, g[f"packet_k{kind}_b{bits}"])


def test_packet_geometry_matches_survey_sizes():
    # Llama-3-8B (8 heads): int8 147472 B, int4 81936 B; Qwen 4 heads int8 73744 B;
    # 70B/TP8 (1 head) int4 10256 B.
    assert codec_oracle.packet_geometry(8, 128, 8)[2] == 147472
    assert codec_oracle.packet_geometry(8, 128, 4)[2] == 81936
    assert codec_oracle.packet_geometry(4, 128, 8)[2] == 73744
    assert codec_oracle.packet_geometry(1, 128, 4)[2] == 10256


@pytest.mark.parametrize("bits", [8, 4])
def test_reciprocal_quantise_matches_division(bits):
    """The device encode replaces (x - low) / scale by (x - low) * fl(1/scale)
    and falls back to the division only within 2^-13 of a half-integer; in
    IEEE fp32 (numpy rounds like the device's _rn intrinsics) that gives the
    same quantised levels as the reference's division on every sample."""
    rng = np.random.default_rng(bits)
    levels = np.float32((1 << bits) - 1)
    n = 1_000_000
    low = rng.standard_normal(n).astype(np.float32) * np.float32(3)
    span = np.abs(rng.standard_normal(n).astype(np.float32)) * np.float32(rng.uniform(1e-6, 20, n).astype(np.float32))
    high = (low + span).astype(np.float32)
    scale = np.maximum(((high - low).astype(np.float32) / levels).astype(np.float32), np.float32(1e-12))
    x = np.clip((low + rng.random(n).astype(np.float32) * (high - low)).astype(np.float32), low, high)
    d = (x - low).astype(np.float32)
    exact = np.rint((d / scale).astype(np.float32))
    y = (d * (np.float32(1) / scale).astype(np.float32)).astype(np.float32)
    near = np.abs((y - np.floor(y)).astype(np.float32) - np.float32(0.5)) < np.float32(2 ** -13)
    fast = np.where(near, exact, np.rint(y))
    assert np.array_equal(fast, exact)
    assert near.mean() < 1e-3


SHAPE_CASES = [(name, tag) for name, e in codec_shapes().items() for tag in e["cases"]]


@pytest.mark.parametrize("name,tag", SHAPE_CASES)
def test_codec_oracle_at_config_shapes(name, tag):
    """The numpy and torch restatements reproduce the reference's own packets
    and decode_into output at the benchmark configs' shapes (4 heads with
    outliers, 8 heads int8 / int4, 1 head int4 over 64 blocks); this is where
    the K-group index depends on the head count."""
    torch = pytest.importorskip("torch")
    e = codec_shapes()[name]
    c = e["cases"][tag]
    src = codec_shape_source(e)
    packet, qb, sb = codec_oracle.encode(src, e["enc_idx"], c["bits"], c["kind"], c["layer"])
    assert (qb, sb, packet.shape[1]) == (c["qb"], c["sb"], c["width"])
    assert sha256(packet) == c["packet_sha256"]
    tpacket, _, _ = codec_oracle.encode_torch(src, e["enc_idx"], c["bits"], c["kind"], c["layer"])
    assert np.array_equal(tpacket, packet)
    dest = np.zeros((e["dst_blocks"], 128, e["heads"], 128), np.uint16)
    codec_oracle.decode_into(packet, dest, e["dst_idx"], c["bits"], c["kind"], qb, sb)
    assert sha256(dest[e["dst_idx"]]) == c["dest_sha256"]
    tdest = torch.zeros((e["dst_blocks"], 128, e["heads"], 128), dtype=torch.bfloat16)
    codec_oracle.decode_into_torch(torch.from_numpy(packet), tdest, torch.tensor(e["dst_idx"]), c["bits"], c["kind"],
                                   qb, sb)
    assert np.array_equal(tdest.view(torch.int16).numpy().view(np.uint16), dest)


@pytest.mark.parametrize("heads", [1, 2])
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("bits", [8, 4])
def test_codec_torch_decode_bit_exact_vs_reference(heads, kind, bits):
    """The torch restatement of decode_into (the CPU baseline's decode) gives
    the reference's own output."""
    torch = pytest.importorskip("torch")
    g = load_codec(heads)
    tag = f"k{kind}_b{bits}"
    dest = torch.zeros((6, 128, heads, 128), dtype=torch.bfloat16)
    codec_oracle.decode_into_torch(torch.from_numpy(g[f"packet_{tag}"]), dest, torch.from_numpy(g["dst_idx"]), bits,
                                   kind, int(g[f"qb_{tag}"]), int(g[f"sb_{tag}"]))
    got = dest.view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got[g["dst_idx"]], g[f"dest_{tag}"])
