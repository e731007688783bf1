"""TEST INFRASTRUCTURE ONLY: ctypes wrapper over the C oracle (gcm_oracle.c).

Used by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline and
reference arm as the checker; the product path never imports it.
"""
from __future__ import annotations

import ctypes as ct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libgcm_oracle.so"

_u8p = ct.POINTER(ct.c_uint8)
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ct.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ct.CDLL(str(LIB_PATH))
        P, U64, U32 = ct.c_void_p, ct.c_uint64, ct.c_uint32
        sig = {
            "orc_aes128_expand": ([P, P], None),
            "orc_aes128_block": ([P, P, P], None),
            "orc_gf_mul": ([P, P, P], None),
            "orc_ghash": ([P, P, U64, P, U64, P], None),
            "orc_aes_ctr": ([P, P, P, U64, P], ct.c_int),
            "orc_keystream": ([P, P, U64, P], ct.c_int),
            "orc_gcm_decrypt_verify": ([P, P, P, P, P, P, U64, P, P, U64], ct.c_int),
            "orc_gcm_verify_xor": ([P, P, P, P, P, P, P, U64, P, P, U64], ct.c_int),
            "orc_gcm_verify_only": ([P, P, P, P, P, U64, P, P, U64], ct.c_int),
            "orc_gcm_encrypt_tag": ([P, P, P, P, P, U64, P, P, U64], ct.c_int),
            "orc_ghash_flags": ([P, P, P, P, P, P, P, P, P, U64, U64, U32], ct.c_int),
            "orc_auth_gate": ([P, P, U64], ct.c_int),
            "orc_derive_transfer_iv": ([P, U64, U64, U64, P], None),
            "orc_build_gcm_aad": ([ct.c_uint8, U32, U32, U64, U64, U64, U64, U64, U64, P], None),
            "orc_record_aligned_bytes": ([U64], U64),
            "orc_record_bytes": ([U64], U64),
            "orc_host_encrypt_record": ([P, P, P, P, U64, P], ct.c_int),
            "orc_host_decrypt_verify": ([P, P, P, P, U64, P, P], ct.c_int),
            "orc_host_batch": ([P, P, P, U64, U64, P, P, U64, ct.c_int, ct.c_int], ct.c_int),
        }
        for name, (args, res) in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = res
    return _lib


def _buf(data) -> np.ndarray:
    return np.frombuffer(bytes(data), dtype=np.uint8).copy()


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ct.c_void_p)


def _words(iv_words) -> np.ndarray:
    return np.asarray(iv_words, dtype=np.uint32)


def aes_block(key: bytes, block: bytes) -> bytes:
    rk = np.zeros(176, np.uint8)
    out = np.zeros(16, np.uint8)
    lib().orc_aes128_expand(_ptr(_buf(key)), _ptr(rk))
    lib().orc_aes128_block(_ptr(rk), _ptr(_buf(block)), _ptr(out))
    return out.tobytes()


def gf_mul(x: bytes, y: bytes) -> bytes:
    out = np.zeros(16, np.uint8)
    lib().orc_gf_mul(_ptr(_buf(x)), _ptr(_buf(y)), _ptr(out))
    return out.tobytes()


def ghash(h: bytes, aad: bytes, c: bytes) -> bytes:
    out = np.zeros(16, np.uint8)
    a = _buf(aad) if aad else None
    lib().orc_ghash(_ptr(_buf(h)), _ptr(a), len(aad or b""), _ptr(_buf(c)), len(c), _ptr(out))
    return out.tobytes()


def keystream(key: bytes, nbytes: int, iv_words) -> bytes:
    out = np.zeros(nbytes, np.uint8)
    assert lib().orc_keystream(_ptr(_buf(key)), _ptr(out), nbytes, _ptr(_words(iv_words))) == 0
    return out.tobytes()


def aes_ctr(data: bytes, key: bytes, iv_words) -> bytes:
    out = np.zeros(len(data), np.uint8)
    assert lib().orc_aes_ctr(_ptr(_buf(data)), _ptr(_buf(key)), _ptr(out), len(data),
                             _ptr(_words(iv_words))) == 0
    return out.tobytes()


def gcm_encrypt_tag(plain: bytes, key: bytes, h: bytes, iv_words, aad: bytes | None):
    c = np.zeros(len(plain), np.uint8)
    tag = np.zeros(16, np.uint8)
    a = _buf(aad) if aad else None
    assert lib().orc_gcm_encrypt_tag(_ptr(_buf(plain)), _ptr(_buf(key)), _ptr(_buf(h)), _ptr(c),
                                     _ptr(tag), len(plain), _ptr(_words(iv_words)), _ptr(a),
                                     len(aad or b"")) == 0
    return c.tobytes(), tag.tobytes()


def gcm_decrypt_verify(c: bytes, key: bytes, h: bytes, tag: bytes, iv_words, aad: bytes | None):
    out = np.zeros(len(c), np.uint8)
    st = np.zeros(1, np.uint32)
    a = _buf(aad) if aad else None
    assert lib().orc_gcm_decrypt_verify(_ptr(_buf(c)), _ptr(_buf(key)), _ptr(_buf(h)),
                                        _ptr(_buf(tag)), _ptr(out), _ptr(st), len(c),
                                        _ptr(_words(iv_words)), _ptr(a), len(aad or b"")) == 0
    return out.tobytes(), int(st[0])


def gcm_verify_xor(c: bytes, key: bytes, h: bytes, tag: bytes, ks: bytes, iv_words, aad):
    out = np.zeros(len(c), np.uint8)
    st = np.zeros(1, np.uint32)
    a = _buf(aad) if aad else None
    assert lib().orc_gcm_verify_xor(_ptr(_buf(c)), _ptr(_buf(key)), _ptr(_buf(h)), _ptr(_buf(tag)),
                                    _ptr(_buf(ks)), _ptr(out), _ptr(st), len(c),
                                    _ptr(_words(iv_words)), _ptr(a), len(aad or b"")) == 0
    return out.tobytes(), int(st[0])


def gcm_verify_only(c: bytes, key: bytes, h: bytes, tag: bytes, iv_words, aad) -> int:
    st = np.zeros(1, np.uint32)
    a = _buf(aad) if aad else None
    assert lib().orc_gcm_verify_only(_ptr(_buf(c)), _ptr(_buf(key)), _ptr(_buf(h)), _ptr(_buf(tag)),
                                     _ptr(st), len(c), _ptr(_words(iv_words)), _ptr(a),
                                     len(aad or b"")) == 0
    return int(st[0])


def ghash_flags(data: bytes, h: bytes, aad, mask, expected, ks, flags: int):
    out = np.zeros(16, np.uint8)
    plain = np.zeros(len(data), np.uint8)
    st = np.zeros(1, np.uint32)
    conv = lambda v: _buf(v) if v else None  # noqa: E731
    assert lib().orc_ghash_flags(_ptr(_buf(data)), _ptr(_buf(h)), _ptr(out), _ptr(conv(aad)),
                                 _ptr(conv(mask)), _ptr(conv(expected)), _ptr(conv(ks)), _ptr(plain),
                                 _ptr(st), len(data), len(aad or b""), flags) == 0
    return out.tobytes(), plain.tobytes(), int(st[0])


def derive_transfer_iv(salt: bytes, ticket: int, block_offset: int = 0, session_nonce: int = 0) -> bytes:
    base = _buf(salt + bytes(12))
    out = np.zeros(16, np.uint8)
    lib().orc_derive_transfer_iv(_ptr(base), session_nonce, ticket, block_offset, _ptr(out))
    return out.tobytes()


def build_gcm_aad(direction, kind, layer, block_id, byte_offset, nbytes, ticket,
                  transfer_offset=0, epoch=0) -> bytes:
    out = np.zeros(64, np.uint8)
    lib().orc_build_gcm_aad(direction, kind, layer, block_id, byte_offset, nbytes, ticket,
                            transfer_offset, epoch, _ptr(out))
    return out.tobytes()


def record_aligned_bytes(count: int) -> int:
    return int(lib().orc_record_aligned_bytes(count))


def record_bytes(count: int) -> int:
    return int(lib().orc_record_bytes(count))


def host_encrypt_record(key: bytes, iv: bytes, aad: bytes | None, plain: bytes) -> bytes:
    rec = np.zeros(record_bytes(len(plain)), np.uint8)
    a = _buf(aad) if aad else None
    assert lib().orc_host_encrypt_record(_ptr(_buf(key)), _ptr(_buf(iv)), _ptr(a), _ptr(_buf(plain)),
                                         len(plain), _ptr(rec)) == 0
    return rec.tobytes()


def host_decrypt_verify(key: bytes, iv: bytes, aad, c: bytes, tag: bytes):
    out = np.zeros(len(c), np.uint8)
    a = _buf(aad) if aad else None
    st = lib().orc_host_decrypt_verify(_ptr(_buf(key)), _ptr(_buf(iv)), _ptr(a), _ptr(_buf(c)),
                                       len(c), _ptr(_buf(tag)), _ptr(out))
    return out.tobytes(), st


def host_batch(key: np.ndarray, ivs: np.ndarray, records: np.ndarray, count: int,
               outs: list[np.ndarray], status: np.ndarray, nthreads: int, encrypt: bool) -> None:
    """records: uint8 [n, stride]; outs: n host arrays (plaintext in/out)."""
    n, stride = records.shape
    ptrs = (ct.c_void_p * n)(*[o.ctypes.data for o in outs])
    rc = lib().orc_host_batch(_ptr(key), _ptr(ivs), _ptr(records), stride, count,
                              ct.cast(ptrs, ct.c_void_p), _ptr(status), n, nthreads, int(encrypt))
    assert rc == 0
