"""Session key agreement primitives on the CPU: the oracle pinned to the
reference's own Monocypher (compiled from its sources into oracle/_ref/), and
the host build of the library's X25519 / BLAKE2b (kx.cuh, the same code the
device kernel runs) checked against the oracle, bit-exact."""
from __future__ import annotations

import random
import shutil
import subprocess
from pathlib import Path

import pytest

from oracle import kx_oracle as kxo

ROOT = Path(__file__).resolve().parents[1]
P25519 = (1 << 255) - 19


def rnd(seed: int, n: int) -> bytes:
    return random.Random(seed).randbytes(n)


def le(v: int) -> bytes:
    return v.to_bytes(32, "little")


SCALARS = [rnd(100 + i, 32) for i in range(24)] + [bytes(32), b"\xff" * 32]
POINTS = ([rnd(200 + i, 32) for i in range(24)]
          + [le(9), le(P25519 - 1), le(P25519 + 1), le(P25519 + 9),        # non-canonical u >= p
             bytes(rnd(7, 31)) + b"\x80", b"\xff" * 32])                    # bit 255 set: masked
LOW_ORDER = [le(0), le(1), le(P25519 - 1 + 1)]                              # shared value is zero
BLAKE_CASES = [(size, rnd(300 + k, klen), rnd(400 + m, mlen))
               for k, (size, klen) in enumerate([(1, 0), (4, 32), (16, 32), (32, 16), (64, 0), (64, 64), (33, 1)])
               for m, mlen in enumerate([0, 1, 63, 127, 128, 129, 255, 256, 257, 1000])]


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path_factory.mktemp("kx") / "kx_driver"
    subprocess.run([cxx, "-O1", "-std=c++17", "-I", str(ROOT / "secure_infer_b200" / "csrc"),
                    str(ROOT / "tests" / "kx_driver.cpp"), "-o", str(exe)], check=True)

    def run(lines: list[str]) -> list[str]:
        out = subprocess.run([str(exe)], input="\n".join(lines) + "\n", capture_output=True, text=True,
                             check=True).stdout
        return out.split("\n")[:len(lines)]
    return run


def h(b: bytes) -> str:
    return b.hex() if b else "-"


def test_oracle_matches_reference_monocypher():
    """The restatement (OpenSSL X25519 + hashlib BLAKE2b) equals the
    reference's vendored Monocypher on every case the tests use."""
    ref = kxo.monocypher()
    if ref is None:
        pytest.skip("oracle/_ref/libmonocypher_ref.so not built (make -C oracle ref REFERENCE_ROOT=...)")
    for s in SCALARS:
        assert kxo.x25519_public(s) == ref.x25519_public(s)
        for u in POINTS:
            assert kxo.x25519(s, u) == ref.x25519(s, u)
        for u in LOW_ORDER:
            assert kxo.x25519(s, u) == ref.x25519(s, u) == bytes(32)
    for size, key, msg in BLAKE_CASES:
        assert kxo.blake2b(msg, size, key) == ref.blake2b(msg, size, key)


def test_x25519_matches_oracle(driver):
    lines = [f"x {s.hex()} {u.hex()}" for s in SCALARS for u in POINTS + LOW_ORDER]
    want = [kxo.x25519(s, u).hex() for s in SCALARS for u in POINTS + LOW_ORDER]
    assert driver(lines) == want
    assert driver([f"p {s.hex()}" for s in SCALARS]) == [kxo.x25519_public(s).hex() for s in SCALARS]


def test_blake2b_matches_oracle(driver):
    lines = [f"b {size} {h(key)} {h(msg)}" for size, key, msg in BLAKE_CASES]
    assert driver(lines) == [kxo.blake2b(msg, size, key).hex() for size, key, msg in BLAKE_CASES]


def test_handshake_derivations_match_oracle(driver):
    """Both ends' derivations: the device's key and proof equal the host's
    expectation, and the host accepts; a wrong proof or challenge is refused."""
    for i in range(8):
        host_secret, dev_secret, challenge = rnd(500 + i, 32), rnd(600 + i, 32), rnd(700 + i, 32)
        host_public, dev_public = kxo.x25519_public(host_secret), kxo.x25519_public(dev_secret)
        shared = kxo.x25519(dev_secret, host_public)
        assert shared == kxo.x25519(host_secret, dev_public)
        key = kxo.derive_key(shared, host_public, dev_public, challenge)
        proof = kxo.derive_proof(key, challenge)
        got = driver([f"d {shared.hex()} {host_public.hex()} {dev_public.hex()} {challenge.hex()}"])[0].split()
        assert got == [key.hex(), proof.hex(), kxo.derive_salt(shared).hex()]
        assert kxo.host_side(host_secret, challenge, dev_public, proof) == (key, kxo.derive_salt(shared))
        bad = bytes([proof[0] ^ 1]) + proof[1:]
        assert kxo.host_side(host_secret, challenge, dev_public, bad) is None
        assert kxo.host_side(host_secret, rnd(800 + i, 32), dev_public, proof) is None
    assert kxo.host_side(rnd(1, 32), rnd(2, 32), le(0), bytes(32)) is None


def test_golden_vectors_from_reference_monocypher(driver):
    """tests/golden/kx_vectors.json holds outputs of the reference's own
    Monocypher (make_kx_golden.py): the oracle and the host build of kx.cuh
    must reproduce every one of them."""
    import json
    g = json.loads((ROOT / "tests" / "golden" / "kx_vectors.json").read_text())
    fx = bytes.fromhex
    for c in g["x25519"]:
        assert kxo.x25519(fx(c["scalar"]), fx(c["u"])).hex() == c["out"]
    assert driver([f"x {c['scalar']} {c['u']}" for c in g["x25519"]]) == [c["out"] for c in g["x25519"]]
    for c in g["public"]:
        assert kxo.x25519_public(fx(c["scalar"])).hex() == c["out"]
    assert driver([f"p {c['scalar']}" for c in g["public"]]) == [c["out"] for c in g["public"]]
    for c in g["blake2b"]:
        assert kxo.blake2b(fx(c["msg"]), c["size"], fx(c["key"])).hex() == c["out"]
    assert driver([f"b {c['size']} {c['key'] or '-'} {c['msg'] or '-'}" for c in g["blake2b"]]) == \
        [c["out"] for c in g["blake2b"]]
    for h in g["handshakes"]:
        shared = fx(h["shared"])
        assert kxo.x25519_public(fx(h["host_secret"])).hex() == h["host_public"]
        assert kxo.x25519(fx(h["host_secret"]), fx(h["device_public"])) == shared
        assert kxo.derive_key(shared, fx(h["host_public"]), fx(h["device_public"]), fx(h["challenge"])).hex() == h["key"]
        got = driver([f"d {h['shared']} {h['host_public']} {h['device_public']} {h['challenge']}"])[0].split()
        assert got == [h["key"], h["proof"], h["salt"]]
        assert kxo.host_side(fx(h["host_secret"]), fx(h["challenge"]), fx(h["device_public"]), fx(h["proof"])) == \
            (fx(h["key"]), fx(h["salt"]))
