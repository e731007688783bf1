"""ctypes binding of the in-tree native library ``_build/libsecure_infer.so``.

The library is the product: there is no Python or CPU fallback.  If it is
missing, ``lib()`` raises ``NativeLibraryMissing`` with the build command.
"""
from __future__ import annotations

import ctypes as ct
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_build" / "libsecure_infer.so"

P, U64, U32, I32, SZ = ct.c_void_p, ct.c_uint64, ct.c_uint32, ct.c_int, ct.c_size_t
PP = ct.POINTER(ct.c_void_p)
U32P = ct.POINTER(ct.c_uint32)
U64P = ct.POINTER(ct.c_uint64)


class NativeLibraryMissing(RuntimeError):
    pass


# name -> (argtypes, restype)
PLUGIN_SIGNATURES = {
    "secure_infer_aicpu_ghash_do": ([P] * 10 + [U64, U64, U32], I32),
    "secure_infer_aicpu_auth_gate_do": ([P, P, P, U64], I32),
    "secure_infer_aicpu_aes_ctr_do": ([P, P, P, P, U64] + [U32] * 4, I32),
    "secure_infer_aicpu_keystream_do": ([P, P, P, U64] + [U32] * 4, I32),
    "secure_infer_aicpu_keystream_batch_do": ([P, P, PP, U32P, U64, U32], I32),
    "secure_infer_aicpu_gcm_decrypt_verify_do": ([P] * 7 + [U64] + [U32] * 4, I32),
    "secure_infer_aicpu_gcm_decrypt_verify_aad_do": ([P] * 7 + [U64] + [U32] * 4 + [P, U64], I32),
    "secure_infer_aicpu_gcm_encrypt_tag_do": ([P] * 6 + [U64] + [U32] * 4 + [P, U64], I32),
    "secure_infer_aicpu_gcm_verify_xor_do": ([P] * 8 + [U64] + [U32] * 4, I32),
    "secure_infer_aicpu_gcm_verify_xor_aad_do": ([P] * 8 + [U64] + [U32] * 4 + [P, U64], I32),
    "secure_infer_aicpu_gcm_verify_only_do": ([P] * 6 + [U64] + [U32] * 4, I32),
    "secure_infer_aicpu_gcm_verify_only_aad_do": ([P] * 6 + [U64] + [U32] * 4 + [P, U64], I32),
    "secure_infer_aicpu_gcm_verify_xor_batch_do": ([P, P, P, PP, PP, PP, PP, PP, PP, U64, U64, U32P, U32], I32),
    "secure_infer_aicpu_gcm_xor_only_do": ([P] * 8 + [U64] + [U32] * 4, I32),
}

HOST_SIGNATURES: dict[str, tuple[list, object]] = {}

_lib: ct.CDLL | None = None


def lib() -> ct.CDLL:
    """Load (once) and return the native library with typed entry points."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is missing; build it with `python -m secure_infer_b200.build`")
        handle = ct.CDLL(str(LIB_PATH))
        for table in (PLUGIN_SIGNATURES, HOST_SIGNATURES):
            for name, (args, res) in table.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue
                fn.argtypes = args
                fn.restype = res
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return [name for name in (*PLUGIN_SIGNATURES, *HOST_SIGNATURES) if hasattr(lib(), name)]
