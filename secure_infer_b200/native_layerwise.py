"""Layerwise authenticated KV transfer over the CUDA C ABI.

Python mirror of the reference's connector-facing objects for this path:

* ``settings`` / ``layer_bits`` -- secure_infer/kv_offload/transport_codec.py:9-19
* ``NativeTransfer.single_layer_kv_transfer`` -- native_layerwise.py:94-130:
  per layer, K then V, every mapped block reloaded through the authenticated
  path.  Instead of one vendor copy per block (``swap_blocks`` interposed by
  the native library) each kind is one staged copy plus one fused kernel.
* ``PackedTransfer.transfer`` (codec packets, transport_codec.py:146-199 /
  pipelined_codec.py:74-139): packets are authenticated, dequantised and
  scattered into the paged cache by the same fused kernel.
* ``wait_for_layer_load`` -- reuse/connector.py:378-410: blocks until the
  layer's records are authenticated (one strict retry on failure), raising
  ``RuntimeError('Packed KV authentication failed')`` like
  pipelined_codec.py:118.
* ``store_layer`` -- writeback (transfer_async D2H + EncodedStore.encode_job):
  gather + quantise + encrypt + tag on the device, host verify into the pool.

PyTorch only supplies tensors and streams; all work goes through
``libsecure_infer.so`` and fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as ct
import json
import math
import os

import torch

from . import _native

CODECS = ("none", "int8", "int4", "mixed")


def settings():
    """transport_codec.py:9-15: (mode, pipeline) from KV_CODEC_CONFIG / KV_CODEC."""
    path = os.environ.get("KV_CODEC_CONFIG", "")
    cfg = json.loads(open(path).read()) if path else {}
    mode = cfg.get("codec", os.environ.get("KV_CODEC", "none"))
    pipeline = bool(cfg.get("pipeline", int(os.environ.get("KV_RECOVERY_PIPELINE", "1"))))
    if mode not in CODECS:
        raise ValueError(mode)
    return mode, pipeline


def layer_bits(mode, layer, layers):
    """transport_codec.py:18-19 (mixed: first ceil(L/3) layers int8, rest int4)."""
    return 8 if mode == "int8" or (mode == "mixed" and layer < math.ceil(layers / 3)) else 4


def packet_bytes(heads: int, bits: int) -> int:
    return int(_native.lib().secure_infer_codec_packet_bytes(heads, bits))


def record_bytes(count: int) -> int:
    return int(_native.lib().secure_infer_record_bytes(count))


def _ptrs(values) -> ct.Array:
    values = list(values)
    return (ct.c_void_p * len(values))(*values)


def _stream(stream=None) -> ct.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ct.c_void_p(s.cuda_stream)


class Session:
    """Process session: key + IV salt on one device (stands in for the device
    key agreement of secure_infer.cpp:449-521, whose outputs are these)."""

    def __init__(self, device: int, key: bytes, salt: bytes):
        if len(key) != 16 or len(salt) != 4:
            raise ValueError("key must be 16 bytes and salt 4 bytes")
        self.lib = _native.lib()
        self.device = device
        self._key = (ct.c_uint8 * 16)(*key)
        self._salt = (ct.c_uint8 * 4)(*salt)
        if self.lib.secure_infer_session_init(device, self._key, self._salt) != 0:
            raise RuntimeError("secure_infer_session_init failed")

    @classmethod
    def key_agreement(cls, device: int) -> "Session":
        """Session whose key and salt come from the X25519 + BLAKE2b handshake
        with the device (secure_infer.cpp:449-521); the key never reaches
        Python.

        Experimental, weak entropy: the GPU has no random source, so the
        device's X25519 secret is a hash of its timers and a counter (the
        reference's AICPU reads /dev/urandom).  A guessed device secret reveals
        the session key.  The recommended path is ``Session(device, key,
        salt)`` with a key from a real key exchange."""
        self = cls.__new__(cls)
        self.lib = _native.lib()
        self.device = device
        if self.lib.secure_infer_session_init_key_agreement(device) != 0:
            raise RuntimeError("secure_infer_session_init_key_agreement failed")
        return self

    def close(self):
        self.lib.secure_infer_session_shutdown()

    def auth_stats(self):
        return auth_stats()


def prefetch_stats() -> dict:
    """Records reloaded from announced entries, reloads that waited for their
    entry, reloads that found announced entries but none matching."""
    r, b, m = ct.c_uint64(), ct.c_uint64(), ct.c_uint64()
    _native.lib().secure_infer_get_transfer_prefetch_stats(ct.byref(r), ct.byref(b), ct.byref(m))
    return dict(ready=r.value, busy=b.value, missing=m.value)


def auth_stats() -> dict:
    """Records verified / rejected / retried since the session started."""
    v, r, t = ct.c_uint64(), ct.c_uint64(), ct.c_uint64()
    _native.lib().secure_infer_get_auth_stats(ct.byref(v), ct.byref(r), ct.byref(t))
    return dict(verified=v.value, rejected=r.value, retried=t.value)


def register_host_range(tensor: torch.Tensor, layer_id: int | None = None, tensor_kind: int | None = None):
    """npu_predict.py:384-408: register a host KV tensor (block = first dim)."""
    lib = _native.lib()
    nbytes = tensor.numel() * tensor.element_size()
    if layer_id is None:
        lib.secure_infer_register_host_range(tensor.data_ptr(), nbytes)
        return
    block_bytes = tensor[0].numel() * tensor.element_size() if tensor.ndim > 0 and tensor.shape[0] > 0 else 0
    lib.secure_infer_register_host_range_ex(tensor.data_ptr(), nbytes, layer_id,
                                            0 if tensor_kind is None else tensor_kind, block_bytes)


class LayerArrays:
    """ctypes arguments of one layer's reload (NativeTransfer.layer_arrays)."""
    __slots__ = ("layer", "srcs", "dsts", "n", "count", "codec", "codec_arg")

    def __init__(self, layer, srcs, dsts, n, count, codec):
        self.layer, self.srcs, self.dsts, self.n, self.count, self.codec = layer, srcs, dsts, n, count, codec
        self.codec_arg = ct.byref(codec) if codec is not None else None


class NativeTransfer:
    """Per-layer reload of mapped blocks (native_layerwise.py:94-130).

    ``single_layer_kv_transfer((host, mapping), destination)``: host is the
    per-layer ``[K, V]`` pinned host tensors ``[num_cpu_blocks, 128, H, D]``,
    mapping an int64 ``[n, 2]`` tensor of (host block, device block), and
    destination the layer's ``[K, V]`` paged cache tensors.  With a codec mode
    the host tensors are packet arrays ``[num_cpu_blocks, width]`` and the
    packets are dequantised into the bf16 destination blocks.
    """

    def __init__(self, mode: str = "none", layers: int = 1, heads: int | None = None):
        self.lib = _native.lib()
        self.mode = mode
        self.layers = layers
        self.heads = heads
        self.layer = 0

    def _sources(self, host, mapping, heads: int, layer: int):
        """(source pointers, record bytes, codec) of one layer's reload: K
        records first, then V, in mapping order."""
        src_idx = mapping[:, 0].tolist()
        if self.mode == "none":
            codec = None
            counts = {src[0].numel() * src.element_size() for src in host}
            if len(counts) != 1:
                raise ValueError("K and V blocks differ in size")
            count = counts.pop()
        else:
            bits = layer_bits(self.mode, layer, self.layers)
            codec = _native.Codec(bits, _native.KIND_KV, heads, layer)
            count = packet_bytes(heads, bits)
            for src in host:
                if src.shape[1] != count:
                    raise ValueError(f"packet width {src.shape[1]} != {count}")
        srcs = []
        for src in host:
            stride = src.stride(0) * src.element_size()
            srcs += [src.data_ptr() + i * stride for i in src_idx]
        return srcs, count, codec

    def single_layer_kv_transfer(self, payload, destination, stream=None):
        """K and V of the layer go out as one reload of 2n records (K records
        first), so both kinds share one staged copy and one fused kernel."""
        host, mapping = payload
        layer = self.layer
        srcs, count, codec = self._sources(host, mapping, destination[0].shape[2], layer)
        dst_idx = mapping[:, 1].tolist()
        dsts = []
        for dst in destination:
            dstride = dst.stride(0) * dst.element_size()
            dsts += [dst.data_ptr() + i * dstride for i in dst_idx]
        rc = self.lib.secure_infer_h2d_reload_layer(layer, _ptrs(srcs), _ptrs(dsts), len(srcs), count,
                                                    ct.byref(codec) if codec else None, 0, None, _stream(stream))
        if rc != 0:
            raise RuntimeError(f"secure_infer_h2d_reload_layer failed for layer {layer}")
        self.layer += 1

    def layer_arrays(self, payload, destination, layer: int) -> "LayerArrays":
        """The C-ABI argument arrays of one layer's reload (K records, then V),
        built once so a caller that reloads many layers back to back (the
        connector's fetch thread) spends no Python time per layer beyond the
        two library calls."""
        host, mapping = payload
        srcs, count, codec = self._sources(host, mapping, destination[0].shape[2], layer)
        dst_idx = mapping[:, 1].tolist()
        dsts = []
        for dst in destination:
            dstride = dst.stride(0) * dst.element_size()
            dsts += [dst.data_ptr() + i * dstride for i in dst_idx]
        return LayerArrays(layer, _ptrs(srcs), _ptrs(dsts), len(srcs), count, codec)

    def reload_arrays(self, a: "LayerArrays", stream: ct.c_void_p) -> None:
        """secure_infer_h2d_reload_layer of prepared arrays on `stream` (a raw
        stream handle)."""
        rc = self.lib.secure_infer_h2d_reload_layer(a.layer, a.srcs, a.dsts, a.n, a.count, a.codec_arg, 0, None,
                                                    stream)
        if rc != 0:
            raise RuntimeError(f"secure_infer_h2d_reload_layer failed for layer {a.layer}")

    def prepare_arrays(self, a: "LayerArrays") -> bool:
        """secure_infer_h2d_prepare_layer (the lookahead) of prepared arrays."""
        rc = self.lib.secure_infer_h2d_prepare_layer(a.layer, a.srcs, a.n, a.count, a.codec_arg)
        if rc < 0:
            raise RuntimeError(f"secure_infer_h2d_prepare_layer failed for layer {a.layer}")
        return rc == 0

    def prepare_layer(self, payload, heads: int, layer: int | None = None) -> bool:
        """Announce the reload of ``payload`` for ``layer`` (default: the next
        layer this object transfers) so its records are encrypted ahead of
        time (secure_infer_h2d_prepare_layer).  Returns whether it was
        scheduled."""
        host, mapping = payload
        layer = self.layer if layer is None else layer
        srcs, count, codec = self._sources(host, mapping, heads, layer)
        rc = self.lib.secure_infer_h2d_prepare_layer(layer, _ptrs(srcs), len(srcs), count,
                                                     ct.byref(codec) if codec else None)
        if rc < 0:
            raise RuntimeError(f"secure_infer_h2d_prepare_layer failed for layer {layer}")
        return rc == 0

    def wait_for_layer_load(self, layer: int):
        if self.lib.secure_infer_recovery_wait_layer_authentication(layer) != 0:
            raise RuntimeError("Packed KV authentication failed")

    def layer_ready_on(self, layer: int, stream=None) -> bool:
        """Make `stream` wait (device side) for the layer's last reload."""
        return self.lib.secure_infer_layer_ready_wait(layer, _stream(stream)) == 0


def store_layer(cache: torch.Tensor, block_ids, host: torch.Tensor, host_ids, *, kind: int, layer: int,
                bits: int = 0, stream=None) -> None:
    """Writeback of blocks ``cache[block_ids]`` into ``host[host_ids]``:
    quantise (bits 8/4) or raw (bits 0), encrypt + tag on the device, verify
    and decrypt on the host.  Completion is joined by ``wait_stores``."""
    lib = _native.lib()
    heads = cache.shape[2]
    cstride = cache.stride(0) * cache.element_size()
    hstride = host.stride(0) * host.element_size()
    srcs = _ptrs(cache.data_ptr() + int(i) * cstride for i in block_ids)
    dsts = _ptrs(host.data_ptr() + int(i) * hstride for i in host_ids)
    codec = _native.Codec(bits, kind, heads, layer)
    if lib.secure_infer_d2h_writeback_layer(srcs, dsts, len(srcs), ct.byref(codec), _stream(stream)) != 0:
        raise RuntimeError("secure_infer_d2h_writeback_layer failed")


def wait_stores() -> None:
    if _native.lib().secure_infer_d2h_wait() != 0:
        raise RuntimeError("async D2H authentication/decrypt failed; cache entry withheld")
