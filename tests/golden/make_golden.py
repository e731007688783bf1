"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the reference checkout and ``cryptography``:

    python tests/golden/make_golden.py --reference <path-to-secure_infer-checkout>

It is never run on the GPU box; the tests only read the files it writes.

Fixtures:
  gcm_kat.json      -- AES-128-GCM known answers produced the way the reference's
                       device KAT does (secure_infer/tests/crypto_smoke.py:39-67):
                       ``cryptography`` AESGCM(key).encrypt(nonce, plain, aad),
                       H = AES-ECB(key, 0^16), IV words = (BE words of nonce, 2),
                       sizes 16, 31, 32768, 262144, 16-byte key, 12-byte nonce,
                       64-byte AAD.  Payloads come from ``det_bytes`` (SHA-256
                       counter stream) so large ones are stored as digests.
  records.json      -- host records (IV from secure_infer.cpp:274-300, AAD from
                       secure_infer.cpp:730-775, record layout :6379-6388) for
                       a few (layer, kind, block, ticket) tuples, encrypted with
                       ``cryptography`` AESGCM (an implementation independent of
                       the oracle's OpenSSL path).
  codec_*.npz       -- outputs of the reference codec itself, imported from the
                       checkout: transport_codec.encode (:22-42) and
                       optimized_decode.decode_into (:5-27) on CPU torch.
  codec_shapes.json -- the same reference encode / decode_into at the shapes of
                       the benchmark configs (4 heads int8 + int4 with 1%
                       outliers at 8 sigma; 8 heads int8 + int4 at the mixed
                       split's layers; 1 head int4 over 64 blocks), stored as
                       SHA-256 digests of the packets and of the decoded
                       blocks.  The source values are regenerated from the
                       stored seed (numpy PCG64 normal draws, RNE to bf16) and
                       pinned by their own digest.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import struct
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def det_bytes(seed: str, n: int) -> bytes:
    out = bytearray()
    counter = 0
    while len(out) < n:
        out += hashlib.sha256(f"{seed}:{counter}".encode()).digest()
        counter += 1
    return bytes(out[:n])


def gcm_kat():
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms, modes
    from cryptography.hazmat.primitives.ciphers.aead import AESGCM

    cases = []
    for count in (16, 31, 32768, 262144):
        key = det_bytes(f"key{count}", 16)
        nonce = det_bytes(f"nonce{count}", 12)
        aad = det_bytes(f"aad{count}", 64)
        plain = det_bytes(f"plain{count}", count)
        protected = AESGCM(key).encrypt(nonce, plain, aad)
        ecb = Cipher(algorithms.AES(key), modes.ECB()).encryptor()
        h = ecb.update(bytes(16)) + ecb.finalize()
        # Also a no-AAD answer (the legacy *_do ABI without AAD).
        protected_noaad = AESGCM(key).encrypt(nonce, plain, None)
        case = dict(count=count, key=key.hex(), nonce=nonce.hex(), aad=aad.hex(), h=h.hex(),
                    iv_words=[*struct.unpack(">III", nonce), 2],
                    plain_seed=f"plain{count}",
                    tag=protected[-16:].hex(), tag_noaad=protected_noaad[-16:].hex(),
                    cipher_sha256=hashlib.sha256(protected[:-16]).hexdigest())
        if count <= 32768:
            case["cipher"] = protected[:-16].hex()
        cases.append(case)
    (HERE / "gcm_kat.json").write_text(json.dumps(cases, indent=1))


def derive_iv(salt: bytes, ticket: int, block_offset: int = 0) -> bytes:
    """secure_infer.cpp:274-300 in GCM mode (session nonce 0, counter base 2)."""
    return salt + struct.pack(">Q", ticket) + struct.pack(">I", block_offset + 2)


def build_aad(direction, kind, layer, block_id, byte_offset, nbytes, ticket, transfer_offset, epoch):
    """secure_infer.cpp:730-775."""
    out = bytearray(64)
    out[0:4] = b"SFAD"
    out[4] = 1
    out[5] = direction
    out[6] = kind & 0xFF
    out[8:12] = struct.pack(">I", layer)
    out[12:20] = struct.pack(">Q", block_id)
    out[20:28] = struct.pack(">Q", byte_offset)
    out[28:36] = struct.pack(">Q", nbytes)
    out[36:44] = struct.pack(">Q", ticket)
    out[44:52] = struct.pack(">Q", transfer_offset)
    out[52:60] = struct.pack(">Q", epoch)
    return bytes(out)


def records():
    from cryptography.hazmat.primitives.ciphers.aead import AESGCM

    key = det_bytes("session-key", 16)
    salt = det_bytes("session-salt", 4)
    rows = []
    for layer, kind, block, ticket, count in ((0, 0, 0, 1, 262144), (3, 1, 17, 99, 73744),
                                              (31, 1, 47, 3072, 10256), (5, 0, 2, 7, 31)):
        plain = det_bytes(f"rec{layer}-{kind}-{block}", count)
        iv = derive_iv(salt, ticket)
        aad = build_aad(1, kind, layer, block, 0, count, ticket, 0, 0)
        protected = AESGCM(key).encrypt(iv[:12], plain, aad)
        aligned = max(32, (count + 31) // 32 * 32)
        record = protected[:-16] + bytes(aligned - count) + protected[-16:] + bytes(16) + aad
        rows.append(dict(layer=layer, kind=kind, block=block, ticket=ticket, count=count,
                         plain_seed=f"rec{layer}-{kind}-{block}", iv=iv.hex(), aad=aad.hex(),
                         record_len=len(record), record_sha256=hashlib.sha256(record).hexdigest(),
                         tag=protected[-16:].hex()))
    (HERE / "records.json").write_text(json.dumps(dict(key=key.hex(), salt=salt.hex(), rows=rows),
                                                  indent=1))


def import_reference_codec(reference: Path):
    """Import the reference codec on CPU with a stub for its NPU-only module."""
    sys.path.insert(0, str(reference))
    stub = types.ModuleType("secure_infer.kv_offload.npu_predict")
    stub._register_host_range = lambda *args, **kwargs: None
    sys.modules["secure_infer.kv_offload.npu_predict"] = stub
    from secure_infer.kv_offload import optimized_decode, transport_codec  # noqa: E402
    return transport_codec, optimized_decode


def kv_values(generator, blocks, heads, outliers):
    import torch
    x = torch.from_numpy(generator.standard_normal((blocks, 128, heads, 128)).astype(np.float32))
    if outliers:
        mask = torch.from_numpy(generator.random(x.shape) < 0.01)
        sign = torch.from_numpy(np.where(generator.random(x.shape) < 0.5, -1.0, 1.0).astype(np.float32))
        x = torch.where(mask, 8.0 * sign, x)
    return x.to(torch.bfloat16)


def codec(reference: Path):
    import torch
    tc, od = import_reference_codec(reference)
    generator = np.random.default_rng(20261201)
    for heads, outliers, enc, dst in ((1, True, [2, 0, 3], [4, 1, 0]), (2, False, [2, 0], [4, 1])):
        source = kv_values(generator, 3 if heads == 2 else 4, heads, outliers)
        enc_idx = torch.tensor(enc)
        dst_idx = torch.tensor(dst)
        out = dict(source=source.view(torch.int16).numpy().view(np.uint16),
                   enc_idx=enc_idx.numpy(), dst_idx=dst_idx.numpy())
        for kind in (0, 1):
            for bits in (8, 4):
                packet, qb, sb = tc.encode(source, enc_idx, bits, kind, layer=5)
                dest = torch.zeros((6, 128, heads, 128), dtype=torch.bfloat16)
                od.decode_into(packet, dest, dst_idx, bits, kind, qb, sb)
                tag = f"k{kind}_b{bits}"
                out[f"packet_{tag}"] = packet.numpy()
                out[f"qb_{tag}"] = np.int64(qb)
                out[f"sb_{tag}"] = np.int64(sb)
                # Blocks outside dst_idx stay zero; store only the written ones.
                out[f"dest_{tag}"] = dest[dst_idx].view(torch.int16).numpy().view(np.uint16)
        np.savez_compressed(HERE / f"codec_h{heads}.npz", **out)
    bits = {mode: [tc.layer_bits(mode, layer, layers) for layers in (28, 32, 40, 80)
                   for layer in range(layers)] for mode in ("int8", "int4", "mixed")}
    (HERE / "layer_bits.json").write_text(json.dumps(bits))


# name, KV heads, 1% outliers at 8 sigma, host blocks, (bits, layer) pairs.
# Encoded host blocks and destination cache blocks are seeded permutations.
CONFIG_SHAPES = (
    ("c3_h4", 4, True, 8, 10, ((8, 3), (4, 3))),
    ("c4_h8", 8, False, 6, 9, ((8, 10), (4, 11))),
    ("c5_h1", 1, False, 64, 80, ((4, 79),)),
)


def config_source(seed: int, blocks: int, heads: int, outliers: bool) -> np.ndarray:
    """float32 KV values [blocks, 128, heads, 128]: N(0,1), optionally with 1%
    of the entries replaced by +-8."""
    g = np.random.default_rng(seed)
    x = g.standard_normal((blocks, 128, heads, 128)).astype(np.float32)
    if outliers:
        mask = g.random(x.shape) < 0.01
        sign = np.where(g.random(x.shape) < 0.5, -1.0, 1.0).astype(np.float32)
        x = np.where(mask, 8.0 * sign, x).astype(np.float32)
    return x


def codec_shapes(reference: Path):
    import torch
    tc, od = import_reference_codec(reference)
    out = {}
    for i, (name, heads, outliers, blocks, dst_blocks, pairs) in enumerate(CONFIG_SHAPES):
        seed = 20261202 + i
        source = torch.from_numpy(config_source(seed, blocks, heads, outliers)).to(torch.bfloat16)
        g = np.random.default_rng(seed + 1000)
        n = min(blocks, 5) if blocks < 64 else blocks
        enc = [int(v) for v in g.permutation(blocks)[:n]]
        dst = [int(v) for v in g.permutation(dst_blocks)[:n]]
        entry = dict(seed=seed, heads=heads, outliers=outliers, blocks=blocks, dst_blocks=dst_blocks,
                     enc_idx=enc, dst_idx=dst,
                     source_sha256=hashlib.sha256(source.view(torch.int16).numpy().tobytes()).hexdigest(),
                     cases={})
        for bits, layer in pairs:
            for kind in (0, 1):
                packet, qb, sb = tc.encode(source, torch.tensor(enc), bits, kind, layer=layer)
                dest = torch.zeros((dst_blocks, 128, heads, 128), dtype=torch.bfloat16)
                od.decode_into(packet, dest, torch.tensor(dst), bits, kind, qb, sb)
                rows = packet.numpy()
                entry["cases"][f"k{kind}_b{bits}"] = dict(
                    bits=bits, kind=kind, layer=layer, qb=int(qb), sb=int(sb), width=int(rows.shape[1]),
                    packet_sha256=hashlib.sha256(rows.tobytes()).hexdigest(),
                    packet_row_sha256=[hashlib.sha256(r.tobytes()).hexdigest()[:16] for r in rows],
                    dest_sha256=hashlib.sha256(dest[torch.tensor(dst)].view(torch.int16).numpy().tobytes()).hexdigest())
        out[name] = entry
    (HERE / "codec_shapes.json").write_text(json.dumps(out, indent=1))


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args()
    gcm_kat()
    records()
    codec(args.reference)
    codec_shapes(args.reference)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
