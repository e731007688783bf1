"""Codec transfer objects of the reference's kv_offload package, over the CUDA C ABI.

* ``EncodedStore``   -- secure_infer/kv_offload/transport_codec.py:45-143.  The
  reference keeps raw bf16 blocks in the host cache and, after a store job's
  D2H copy, encodes them on a CPU thread into per-(layer, kind, bits) packet
  arrays, publishing the job only once encoding is done.  Here the packets are
  produced on the GPU (gather + quantise + encrypt + tag) and verified and
  decrypted by the host into the same arrays; the job is published only after
  that verification (two-phase completion).  Slot versions guard every read:
  a slot rewritten by a later store is stale until that store is published.
* ``PackedTransfer`` -- transport_codec.py:146-199.  A layer's K and V packets
  for the mapping's CPU slots are authenticated, dequantised and scattered into
  the paged cache by one ``secure_infer_h2d_reload_layer`` call (the reference
  copies them with ``swap_blocks``, waits for authentication and then decodes).
* ``PipelinedTransfer`` -- pipelined_codec.py:11-151.  Submission and recovery
  on separate threads: the recovery thread waits for each layer's
  authentication and hands ``on_ready(layer, event, start)`` a CUDA event
  recorded after the layer's fused kernel; an authentication failure reaches
  ``on_error``.  The reference's separate decode launch on a recovery stream
  is part of the fused kernel here.
"""
from __future__ import annotations

import ctypes as ct
import queue
import threading
import time

import torch

from . import _native
from .native_layerwise import _ptrs, _stream, layer_bits, packet_bytes, settings


class EncodedStore:
    """Packet arrays ``arrays[(layer, kind, bits)] = (pinned [slots, width],
    qb, sb)`` filled by GPU writeback, with per-slot versions."""

    def __init__(self, num_slots: int, layers: int, heads: int, mode: str | None = None):
        self.lib = _native.lib()
        self.num_slots = num_slots
        self.layers = layers
        self.heads = heads
        self.mode = mode if mode is not None else settings()[0]
        self.lock = threading.RLock()
        self.versions = [0] * num_slots
        self.arrays: dict[tuple[int, int, int], tuple[torch.Tensor, int, int]] = {}
        self.ready: dict[tuple[int, int, int], list] = {}
        self.jobs: dict[object, dict] = {}
        self.pending: list[object] = []

    def _array(self, layer: int, kind: int, bits: int):
        key = (layer, kind, bits)
        if key not in self.arrays:
            width = packet_bytes(self.heads, bits)
            cpu = torch.zeros((self.num_slots, width), dtype=torch.uint8).pin_memory()
            from .native_layerwise import register_host_range
            register_host_range(cpu, layer, kind)
            elements = 128 * self.heads * 128
            self.arrays[key] = (cpu, elements * bits // 8, elements // 64 * 4)
            self.ready[key] = [None] * self.num_slots
        return self.arrays[key]

    def submit(self, job, slot_ids) -> None:
        """transport_codec.py:55-64: a store job for these CPU slots; their
        versions advance, so older packets in them are stale from now on."""
        ids = [int(i) for i in slot_ids]
        with self.lock:
            for i in ids:
                self.versions[i] += 1
            self.jobs[job] = dict(ids=ids, versions=tuple(self.versions[i] for i in ids), mode=self.mode,
                                  keys=set())

    def store_layer(self, job, layer: int, caches, block_ids, stream=None) -> None:
        """Device writeback of one layer of a submitted job: the K and V blocks
        ``caches[k][block_ids]`` become packets in the job's slots."""
        entry = self.jobs[job]
        ids, mode = entry["ids"], entry["mode"]
        if mode == "none":
            raise ValueError("EncodedStore holds codec packets; KV_CODEC=none stores raw blocks")
        bits = layer_bits(mode, layer, self.layers)
        srcs, dsts = [], []
        for kind, cache in enumerate(caches):
            if cache.shape[2] != self.heads:
                raise ValueError("cache heads differ from the store's")
            cpu, _, _ = self._array(layer, kind, bits)
            cstride = cache.stride(0) * cache.element_size()
            srcs += [cache.data_ptr() + int(b) * cstride for b in block_ids]
            dsts += [cpu.data_ptr() + i * cpu.shape[1] for i in ids]
        codec = _native.Codec(bits, _native.KIND_KV, self.heads, layer)
        if self.lib.secure_infer_d2h_writeback_layer(_ptrs(srcs), _ptrs(dsts), len(srcs), ct.byref(codec),
                                                     _stream(stream)) != 0:
            raise RuntimeError("secure_infer_d2h_writeback_layer failed")
        with self.lock:
            entry["keys"].update((layer, kind, bits) for kind in range(len(caches)))
            if job not in self.pending:
                self.pending.append(job)

    def finished(self) -> list:
        """Jobs whose packets are verified on the host, published now
        (transport_codec.py:84-100).  Raises if a packet failed verification."""
        with self.lock:
            if not self.pending:
                return []
            if self.lib.secure_infer_d2h_wait() != 0:
                raise RuntimeError("async D2H authentication/decrypt failed; cache entry withheld")
            done, self.pending = self.pending, []
            for job in done:
                entry = self.jobs.pop(job)
                for key in entry["keys"]:
                    for i, v in zip(entry["ids"], entry["versions"]):
                        # A later store of the slot keeps it stale.
                        if self.versions[i] == v:
                            self.ready[key][i] = v
            return done

    def wait(self, jobs) -> None:
        """transport_codec.py:107-110."""
        if any(job in self.pending for job in jobs):
            self.finished()

    def get(self, layer: int, kind: int, bits: int, ids):
        """transport_codec.py:112-118: the packet array for a reload; every
        requested slot must hold the latest published packets."""
        key = (layer, kind, bits)
        with self.lock:
            if key not in self.arrays:
                raise RuntimeError("No encoded cache; reload must never encode")
            if any(self.ready[key][int(i)] != self.versions[int(i)] for i in ids):
                raise RuntimeError("Encoded cache missing or stale; reload must never encode")
            return self.arrays[key]


class PackedTransfer:
    """One layer per ``transfer`` call (transport_codec.py:146-199):
    ``payload = (host, mapping)`` with mapping rows (CPU slot, GPU block),
    ``destinations = [K, V]`` paged caches."""

    def __init__(self, store: EncodedStore, mode: str | None = None, layers: int | None = None):
        self.lib = _native.lib()
        self.store = store
        self.mode = mode if mode is not None else store.mode
        self.layers = layers if layers is not None else store.layers
        self.layer = 0
        self.records: list[dict] = []

    def transfer(self, payload, destinations, stream=None):
        host, mapping = payload
        layer = self.layer
        src_ids = [int(i) for i in mapping[:, 0].tolist()]
        dst_ids = [int(i) for i in mapping[:, 1].tolist()]
        started = time.monotonic_ns()
        srcs, dsts = [], []
        if self.mode == "none":
            count = host[0][0].numel() * host[0].element_size()
            codec = None
            for src, dst in zip(host, destinations):
                sstride = src.stride(0) * src.element_size()
                srcs += [src.data_ptr() + i * sstride for i in src_ids]
                dstride = dst.stride(0) * dst.element_size()
                dsts += [dst.data_ptr() + i * dstride for i in dst_ids]
        else:
            bits = layer_bits(self.mode, layer, self.layers)
            count = 0
            for kind, dst in enumerate(destinations):
                cpu, _, _ = self.store.get(layer, kind, bits, src_ids)
                count = cpu.shape[1]
                srcs += [cpu.data_ptr() + i * count for i in src_ids]
                dstride = dst.stride(0) * dst.element_size()
                dsts += [dst.data_ptr() + i * dstride for i in dst_ids]
            codec = _native.Codec(bits, _native.KIND_KV, destinations[0].shape[2], layer)
        rc = self.lib.secure_infer_h2d_reload_layer(layer, _ptrs(srcs), _ptrs(dsts), len(srcs), count,
                                                    ct.byref(codec) if codec is not None else None, 0, None,
                                                    _stream(stream))
        if rc != 0:
            raise RuntimeError(f"secure_infer_h2d_reload_layer failed for layer {layer}")
        self.records.append(dict(layer=layer, blocks=len(src_ids), wire_bytes=len(srcs) * count,
                                 original_bytes=sum(len(src_ids) * d[0].numel() * d.element_size()
                                                    for d in destinations),
                                 host_elapsed_ms=(time.monotonic_ns() - started) / 1e6))
        self.layer += 1
        return layer

    def wait_auth(self, layer: int) -> int:
        return int(self.lib.secure_infer_recovery_wait_layer_authentication(layer))

    def wait_for_layer_load(self, layer: int) -> None:
        if self.wait_auth(layer) != 0:
            raise RuntimeError("Packed KV authentication failed")


class PipelinedTransfer(PackedTransfer):
    """pipelined_codec.py:11-151: ``start_request`` starts the recovery
    thread, ``transfer`` submits a layer and queues it, the recovery thread
    waits for its authentication and calls ``on_ready(layer, event, start)``
    with a CUDA event recorded after the layer's fused kernel (a consumer
    stream waits on it before attention), and ``finish_request`` joins."""

    def start_request(self, request_id, mode, layers, on_ready, on_error):
        self.request_id = request_id
        self.mode = mode
        self.layers = layers
        self.layer = 0
        self.on_ready = on_ready
        self.on_error = on_error
        self.recovery_error = None
        self.pending = queue.Queue(maxsize=2)
        self.worker = threading.Thread(target=self._recover_loop, name="kv-recovery", daemon=True)
        self.worker.start()

    def _put(self, value):
        while True:
            if self.recovery_error is not None:
                raise RuntimeError(self.recovery_error)
            try:
                self.pending.put(value, timeout=0.1)
                return
            except queue.Full:
                pass

    def transfer(self, payload, destinations, stream=None):
        start = time.monotonic_ns()
        layer = super().transfer(payload, destinations, stream)
        ready = torch.cuda.Event()
        ready.record(stream if stream is not None else torch.cuda.current_stream())
        self._put(dict(layer=layer, event=ready, start=start))
        return layer

    def _recover_loop(self):
        try:
            while True:
                task = self.pending.get()
                if task is None:
                    return
                if self.wait_auth(task["layer"]) != 0:
                    raise RuntimeError("Packed KV authentication failed")
                self.on_ready(task["layer"], task["event"], task["start"])
        except BaseException as error:   # noqa: BLE001 -- reported to the caller
            self.recovery_error = repr(error)
            self.on_error(self.recovery_error)

    def finish_request(self, timeout: float = 120.0):
        if getattr(self, "worker", None) is None:
            return
        self._put(None)
        self.worker.join(timeout=timeout)
        if self.worker.is_alive():
            raise RuntimeError("KV recovery submitter timeout")
        self.worker = None
        if self.recovery_error is not None:
            raise RuntimeError(self.recovery_error)
