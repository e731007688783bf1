"""ctypes binding of the in-tree native library ``_build/libsecure_infer.so``.

The library is the product: there is no Python or CPU fallback.  If it is
missing, ``lib()`` raises ``NativeLibraryMissing`` with the build command.
"""
from __future__ import annotations

import ctypes as ct
import os
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
    "secure_infer_aicpu_key_agreement_do": ([P] * 7, I32),
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
    "secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do": ([P] * 7 + [U64] + [U32] * 4 + [P, U64], I32),
}

CHARP = ct.c_char_p
HOST_SIGNATURES: dict[str, tuple[list, object]] = {
    "secure_infer_session_init": ([I32, P, P], I32),
    "secure_infer_session_init_key_agreement": ([I32], I32),
    "secure_infer_session_shutdown": ([], I32),
    "secure_infer_register_host_range": ([P, SZ], None),
    "secure_infer_register_host_range_ex": ([P, SZ, U32, U32, SZ], None),
    "secure_infer_is_registered_host_range": ([P, SZ], I32),
    "secure_infer_host_pool_info": ([ct.POINTER(U32), ct.POINTER(I32), U32, ct.POINTER(U32)], I32),
    "secure_infer_set_layer_sm_limit": ([U32], U32),
    "secure_infer_new_transfer_ticket": ([], U64),
    "secure_infer_derive_transfer_iv": ([P, U64, U64, P], I32),
    "secure_infer_build_gcm_aad": ([P, SZ, ct.c_uint8, U64, U64, P], I32),
    "secure_infer_record_bytes": ([U64], U64),
    "secure_infer_h2d_encrypt_records": ([PP, U64, U32, P, U64, U64P], I32),
    "secure_infer_codec_packet_bytes": ([U32, U32], U64),
    "secure_infer_reload_records": ([U32, P, U64, U64, U32, U64P, PP, P, P, P, P, P], I32),
    "secure_infer_keystream_records": ([U64P, U32, U64, P, P], I32),
    "secure_infer_verify_records": ([U32, P, U64, U64, U32, U64P, PP, P, P, P, P], I32),
    "secure_infer_h2d_reload_layer": ([U32, PP, PP, U32, U64, P, I32, U64P, P], I32),
    "secure_infer_h2d_prepare_layer": ([U32, PP, U32, U64, P], I32),
    "secure_infer_h2d_reload_layers_async": ([U32, U32, PP, PP, U32, U64P, P, I32, P], I32),
    "secure_infer_h2d_reload_layers_join": ([], I32),
    "secure_infer_layer_ready_wait": ([U32, P], I32),
    "secure_infer_h2d_layer_group_begin": ([SZ], I32),
    "secure_infer_h2d_layer_group_end": ([], I32),
    "secure_infer_h2d_submit": ([P, SZ, P, SZ, P], I32),
    "secure_infer_recovery_wait_layer_authentication": ([U32], I32),
    "secure_infer_recovery_set_job_id": ([U64], None),
    "secure_infer_recovery_wait_job_authentication": ([U64], I32),
    "secure_infer_d2h_batch_begin": ([SZ], I32),
    "secure_infer_d2h_group_begin": ([SZ], I32),
    "secure_infer_d2h_submit": ([P, P, SZ, P], I32),
    "secure_infer_d2h_group_end": ([], I32),
    "secure_infer_d2h_batch_device_barrier": ([], I32),
    "secure_infer_d2h_batch_end": ([], I32),
    "secure_infer_d2h_writeback_layer": ([PP, PP, U32, P, P], I32),
    "secure_infer_d2h_wait": ([], I32),
    "secure_infer_writeback_records": ([PP, PP, U32, P, P, U64, U64P, P], I32),
    "secure_infer_kernel_profile_enable": ([I32], I32),
    "secure_infer_kernel_profile_collect": ([ct.POINTER(ct.c_double), U64P, U32], I32),
    "secure_infer_kernel_name": ([U32], ct.c_char_p),
    "secure_infer_invalidate_transfer_prefetches": ([], None),
    "secure_infer_retire_transfer_prefetches": ([], None),
    "secure_infer_get_transfer_prefetch_stats": ([U64P] * 3, None),
    "secure_infer_get_gcm_keystream_stats": ([U64P] * 7, None),
    "secure_infer_get_npu_keystream_stats": ([U64P] * 3, None),
    "secure_infer_get_npu_keystream_pool_stats": ([U64P] * 2, None),
    "secure_infer_count_ready_unconsumed_gcm_tickets": ([], U64),
    "secure_infer_flush_completed_h2d_profile": ([], I32),
    "secure_infer_drain_h2d_profile_after_job": ([], I32),
    "secure_infer_get_auth_stats": ([U64P] * 3, None),
    "secure_infer_arm_tamper": ([U32, U64, U32], None),
}


class Codec(ct.Structure):
    """secure_infer_codec (include/secure_infer.h)."""
    _fields_ = [("bits", ct.c_uint32), ("kind", ct.c_uint32), ("heads", ct.c_uint32), ("layer", ct.c_uint32)]


# SECURE_INFER_KIND_KV: a reload of 2n records, K packets first, V packets after.
KIND_KV = 2

_lib: ct.CDLL | None = None


def _preloaded() -> ct.CDLL | None:
    """The process namespace, when libsecure_infer.so is already in it (for
    example LD_PRELOADed, as the reference's run.sh:66 does): the symbols are
    then bound through ``ctypes.CDLL(None)`` like the reference's Python side
    (npu_predict.py:158-254).  SECURE_INFER_USE_PRELOADED=0 disables this."""
    if os.environ.get("SECURE_INFER_USE_PRELOADED", "1") == "0":
        return None
    proc = ct.CDLL(None)
    needed = ("secure_infer_session_init", "secure_infer_h2d_reload_layer", "secure_infer_aicpu_ghash_do")
    return proc if all(hasattr(proc, name) for name in needed) else None


def lib() -> ct.CDLL:
    """Load (once) and return the native library with typed entry points."""
    global _lib
    if _lib is None:
        handle = _preloaded()
        if handle is None:
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


def host_pool_info() -> dict:
    """This rank's host worker pool: OpenSSL worker threads (the calling
    thread encrypts as well), the CPUs of the rank's slice and whether the
    workers are pinned to them."""
    threads, pinned = U32(), U32()
    cpus = (I32 * 1024)()
    n = lib().secure_infer_host_pool_info(ct.byref(threads), cpus, 1024, ct.byref(pinned))
    return {"threads": int(threads.value), "cpus": list(cpus[:max(0, min(n, 1024))]), "pinned": bool(pinned.value)}


def exported_symbols() -> list[str]:
    return [name for name in (*PLUGIN_SIGNATURES, *HOST_SIGNATURES) if hasattr(lib(), name)]
