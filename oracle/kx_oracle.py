"""TEST INFRASTRUCTURE ONLY: CPU oracle for the session key agreement.

Restates the handshake of secure_infer/native/secure_infer.cpp:449-521 (host)
and secure_infer/native/kernels/aicpu/key_agreement.aicpu:9-48 (device) over
Python's ``cryptography`` X25519 (OpenSSL, RFC 7748) and ``hashlib.blake2b``
(RFC 7693).  The reference computes both primitives with the Monocypher copy
vendored beside its device kernel (kernels/aicpu/monocypher/monocypher.c,
"Monocypher version __git__"); ``monocypher()`` loads that file compiled
from the reference's sources into oracle/_ref/ (``make -C oracle ref``) when it
has been built, so the tests can pin this restatement to the reference's own
code.  Used by tests/ only; the product path never imports it.
"""
from __future__ import annotations

import ctypes as ct
import hashlib
from pathlib import Path

from cryptography.hazmat.primitives import serialization
from cryptography.hazmat.primitives.asymmetric import x25519 as _x25519

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / "_ref" / "libmonocypher_ref.so"

# secure_infer.cpp:459 / key_agreement.aicpu:18 and secure_infer.cpp:494.
INFO = b"SecureInfer X25519 BLAKE2b test v1"
SALT_LABEL = b"SecureInfer IV salt v1"


def x25519(secret: bytes, peer_public: bytes) -> bytes:
    """crypto_x25519 (RFC 7748 section 5): the raw shared value.  OpenSSL
    refuses the all-zero result of a low-order peer point, which the reference
    rejects too (secure_infer.cpp:486, key_agreement.aicpu:32-34); it is
    returned here as 32 zero bytes."""
    key = _x25519.X25519PrivateKey.from_private_bytes(secret)
    try:
        return key.exchange(_x25519.X25519PublicKey.from_public_bytes(peer_public))
    except ValueError:
        return bytes(32)


def x25519_public(secret: bytes) -> bytes:
    """crypto_x25519_public_key: the scalar times the base point u = 9."""
    return _x25519.X25519PrivateKey.from_private_bytes(secret).public_key().public_bytes(
        serialization.Encoding.Raw, serialization.PublicFormat.Raw)


def blake2b(data: bytes, size: int, key: bytes = b"") -> bytes:
    return hashlib.blake2b(data, digest_size=size, key=key).digest()


def derive_key(shared: bytes, host_public: bytes, device_public: bytes, challenge: bytes) -> bytes:
    """secure_infer.cpp:487-492 / key_agreement.aicpu:37-42: BLAKE2b-128 keyed
    by the shared value over info || host public || device public || challenge."""
    return blake2b(INFO + host_public + device_public + challenge, 16, shared)


def derive_proof(key: bytes, challenge: bytes) -> bytes:
    """secure_infer.cpp:493 / key_agreement.aicpu:43: BLAKE2b-256 keyed by the
    session key over the challenge."""
    return blake2b(challenge, 32, key)


def derive_salt(shared: bytes) -> bytes:
    """secure_infer.cpp:494-495: the 4-byte IV salt, BLAKE2b-32 keyed by the
    shared value over its label."""
    return blake2b(SALT_LABEL, 4, shared)


def host_side(secret: bytes, challenge: bytes, device_public: bytes, proof: bytes):
    """The host's checks after the device answered (secure_infer.cpp:485-499):
    returns (key, salt), or None when the shared value is zero or the proof
    does not match."""
    host_public = x25519_public(secret)
    shared = x25519(secret, device_public)
    if shared == bytes(32):
        return None
    key = derive_key(shared, host_public, device_public, challenge)
    if derive_proof(key, challenge) != proof:
        return None
    return key, derive_salt(shared)


class Monocypher:
    """ctypes view of the reference's Monocypher built in oracle/_ref/."""

    def __init__(self, path: Path = REF_LIB):
        self.lib = ct.CDLL(str(path))
        u8p, sz = ct.c_char_p, ct.c_size_t
        self.lib.crypto_x25519.argtypes = [ct.c_void_p, u8p, u8p]
        self.lib.crypto_x25519_public_key.argtypes = [ct.c_void_p, u8p]
        self.lib.crypto_blake2b_keyed.argtypes = [ct.c_void_p, sz, u8p, sz, u8p, sz]
        for name in ("crypto_x25519", "crypto_x25519_public_key", "crypto_blake2b_keyed"):
            getattr(self.lib, name).restype = None

    def x25519(self, secret: bytes, peer_public: bytes) -> bytes:
        out = ct.create_string_buffer(32)
        self.lib.crypto_x25519(out, secret, peer_public)
        return out.raw

    def x25519_public(self, secret: bytes) -> bytes:
        out = ct.create_string_buffer(32)
        self.lib.crypto_x25519_public_key(out, secret)
        return out.raw

    def blake2b(self, data: bytes, size: int, key: bytes = b"") -> bytes:
        out = ct.create_string_buffer(size)
        self.lib.crypto_blake2b_keyed(out, size, key, len(key), data, len(data))
        return out.raw


def monocypher() -> Monocypher | None:
    """The reference's Monocypher when oracle/_ref/ holds a build of it."""
    return Monocypher() if REF_LIB.exists() else None
