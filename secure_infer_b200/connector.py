"""Worker side of the reference's KV reload connector, on CUDA.

Mirrors ``RuntimeWorker`` of secure_infer/reuse/connector.py for one process
and one GPU, over the per-layer C ABI instead of interposed vendor copies:

* ``start_load`` -- start_kv_transfers (:333-372): records a producer event on
  the caller's stream and starts the request's fetch thread.
* ``_fetch`` / ``_fetch_serialized`` -- fetch / fetch_serialized (:222-331):
  one request at a time (``submission_lock``), the load stream waits for the
  producer event, then every layer is reloaded on the load stream (K and V in
  one ``secure_infer_h2d_reload_layer``).  The next layer is announced before
  each reload (``secure_infer_h2d_prepare_layer``), the CUDA form of the
  reference's history-predicted CPU pre-encryption.  An observer thread
  (observe_layers) waits for each layer's authentication, with its one strict
  retry, and marks the layer authenticated.
* ``wait_for_layer_load`` -- :374-410: every request being consumed must have
  authenticated KV for the layer; the compute stream then waits on the
  layer's CUDA event, so device ordering, not a host synchronize, makes the
  KV visible to attention.  A failure raises ``RuntimeError``.
* ``get_finished`` -- take_secure_store_metadata (:412-420): requests whose
  fetch is done, raising if any failed.

The scheduler side of the reference connector (request admission, TPSR/Cake
cost models, entry gate) stays with the serving engine.
"""
from __future__ import annotations

import ctypes as ct
import itertools
import threading
import time

import numpy as np
import torch

from . import _native
from .native_layerwise import NativeTransfer, settings


class LayerwiseReloader:
    """``names[l]`` is layer l's attention name; ``kv_caches[l] = [K, V]``
    paged device caches ``[blocks, 128, heads, 128]``; ``cpu_tensors[l] =
    [K, V]`` host pools (raw blocks for ``KV_CODEC=none``, packet arrays for
    the codecs) registered with ``register_host_range``."""

    _jobs = itertools.count(1)

    def __init__(self, names, kv_caches, cpu_tensors, mode: str | None = None, lookahead: bool = True,
                 timeout: float = 120.0, native_loop: bool = False, host_gate: bool = True):
        if not (len(names) == len(kv_caches) == len(cpu_tensors)):
            raise ValueError("names, kv_caches and cpu_tensors differ in length")
        self.lib = _native.lib()
        self.names = list(names)
        self.kv_caches = kv_caches
        self.cpu_tensors = cpu_tensors
        self.mode = mode if mode is not None else settings()[0]
        self.lookahead = lookahead
        self.timeout = timeout
        # native_loop: run each request's layer loop on a library thread
        # (secure_infer_h2d_reload_layers_async) instead of the fetch thread.
        # Measured with an attention stand-in, the fetch thread's loop
        # overlapped better, so it is the default.
        self.native_loop = native_loop
        # host_gate: wait_for_layer_load returns only once the layer's
        # authentication is known on the host, as the reference does.  With
        # host_gate=False it returns once the layer is submitted and gates the
        # compute stream on the device alone: records that fail verification
        # are already zero when the layer's event fires, and the failure is
        # raised by a later wait, get_finished() or the last layer.
        self.host_gate = host_gate
        self.device = kv_caches[0][0].device
        self.heads = kv_caches[0][0].shape[2]
        # High priority: attention waits on this stream's reloads, so their
        # kernels are scheduled ahead of normal-priority compute.
        self.load_stream = torch.cuda.Stream(device=self.device, priority=-1)
        self.lock = threading.Condition()
        self.submission_lock = threading.Lock()
        self.load_jobs: dict = {}
        self.consuming: dict = {}
        self.newly_done: set = set()
        self.load_failure: str | None = None

    # ---------------------------------------------------------------- start
    def start_load(self, req_id, source_blocks, dest_blocks) -> None:
        """Reload host blocks ``source_blocks`` into device blocks
        ``dest_blocks`` for every layer of request ``req_id``."""
        if len(source_blocks) != len(dest_blocks):
            raise ValueError("source and destination block lists differ in length")
        pool = min(int(t.shape[0]) for pair in self.cpu_tensors for t in pair)
        cache = min(int(t.shape[0]) for pair in self.kv_caches for t in pair)
        if any(not 0 <= int(b) < pool for b in source_blocks) or any(not 0 <= int(b) < cache for b in dest_blocks):
            raise ValueError("block index outside the host pool or the device cache")
        if req_id in self.load_jobs:
            raise ValueError(f"request {req_id!r} is already loading")
        producer = torch.cuda.Event()
        producer.record(torch.cuda.current_stream(self.device))
        n = len(self.names)
        state = dict(source=list(source_blocks), destination=list(dest_blocks), done=False, error=None,
                     producer_event=producer, submitted=[False] * n, authenticated=[False] * n,
                     ready_events=[None] * n, submissions_done=False)
        self.load_jobs[req_id] = state
        self.consuming[req_id] = state
        state["thread"] = threading.Thread(target=self._fetch, args=(req_id, state), daemon=True)
        state["thread"].start()

    # ---------------------------------------------------------------- fetch
    def _fetch(self, req_id, state):
        with self.submission_lock:
            try:
                if self.load_failure is not None:
                    raise RuntimeError(self.load_failure)
                self._fetch_serialized(req_id, state)
            except BaseException as error:   # noqa: BLE001 -- reported to the waiting layers
                with self.lock:
                    state["error"] = state["error"] or repr(error)
                    self.lock.notify_all()
            finally:
                with self.lock:
                    if state["error"]:
                        self.load_failure = state["error"]
                    state["done"] = True
                    self.newly_done.add(req_id)
                    self.lock.notify_all()

    def _observe_layers(self, state):
        """observe_layers: authentication of each submitted layer, in order."""
        try:
            for layer in range(len(self.names)):
                with self.lock:
                    while not state["submitted"][layer] and not state["error"] and not state["submissions_done"]:
                        self.lock.wait(timeout=1.0)
                    if state["error"] or not state["submitted"][layer]:
                        return
                rc = self.lib.secure_infer_recovery_wait_layer_authentication(layer)
                with self.lock:
                    if rc != 0:
                        state["error"] = state["error"] or "Packed KV authentication failed"
                    else:
                        state["authenticated"][layer] = True
                    self.lock.notify_all()
                if rc != 0:
                    return
        except BaseException as error:   # noqa: BLE001
            with self.lock:
                state["error"] = state["error"] or repr(error)
                self.lock.notify_all()

    def _fetch_serialized(self, req_id, state):
        torch.cuda.set_device(self.device)
        mapping = torch.from_numpy(np.column_stack((state["source"], state["destination"])).astype(np.int64))
        transfer = NativeTransfer(self.mode, layers=len(self.names), heads=self.heads)
        self.lib.secure_infer_recovery_set_job_id(next(self._jobs))
        self.load_stream.wait_event(state["producer_event"])
        observer = threading.Thread(target=self._observe_layers, args=(state,), daemon=True)
        observer.start()
        native = None
        try:
            # Every layer's argument arrays are built before the first reload.
            arrays = [transfer.layer_arrays((self.cpu_tensors[layer], mapping), self.kv_caches[layer], layer)
                      for layer in range(len(self.names))]
            stream = ct.c_void_p(self.load_stream.cuda_stream)
            if self.native_loop and hasattr(self.lib, "secure_infer_h2d_reload_layers_async"):
                # The layer loop runs on a library thread: no reload waits for
                # the interpreter while the model thread launches attention.
                # Each layer's authentication wait and device-side release
                # block until that layer has been submitted.
                native = self._start_native_loop(arrays, stream)
                with self.lock:
                    state["native"] = True
                    state["submitted"] = [True] * len(self.names)
                    self.lock.notify_all()
                return
            with torch.cuda.stream(self.load_stream):
                for layer in range(len(self.names)):
                    with self.lock:
                        if state["error"]:
                            raise RuntimeError(state["error"])
                    if self.lookahead and layer + 1 < len(self.names):
                        transfer.prepare_arrays(arrays[layer + 1])
                    transfer.reload_arrays(arrays[layer], stream)
                    ready = torch.cuda.Event()
                    ready.record(self.load_stream)
                    with self.lock:
                        state["ready_events"][layer] = ready
                        state["submitted"][layer] = True
                        self.lock.notify_all()
        except BaseException as error:   # noqa: BLE001 -- the first failure is the one reported
            with self.lock:
                state["error"] = state["error"] or repr(error)
                self.lock.notify_all()
            raise
        finally:
            with self.lock:
                state["submissions_done"] = True
                self.lock.notify_all()
            observer.join(timeout=self.timeout)
            if native is not None:
                if self.lib.secure_infer_h2d_reload_layers_join() != 0:
                    with self.lock:
                        state["error"] = state["error"] or "secure_infer_h2d_reload_layers_async: a reload failed"
            elif self.lookahead:
                self.lib.secure_infer_retire_transfer_prefetches()
            with self.lock:
                if observer.is_alive():
                    state["error"] = state["error"] or "authentication observer timeout"
                elif not state["error"] and not all(state["authenticated"]):
                    state["error"] = "layers left unauthenticated"

    def _start_native_loop(self, arrays, stream):
        """secure_infer_h2d_reload_layers_async over the request's layers; the
        argument arrays are kept alive with the request state."""
        n = arrays[0].n
        srcs = (ct.c_void_p * (n * len(arrays)))()
        dsts = (ct.c_void_p * (n * len(arrays)))()
        for i, a in enumerate(arrays):
            if a.n != n:
                raise ValueError("every layer of a request reloads the same blocks")
            srcs[i * n:(i + 1) * n] = a.srcs[:]
            dsts[i * n:(i + 1) * n] = a.dsts[:]
        counts = (ct.c_uint64 * len(arrays))(*[a.count for a in arrays])
        codecs = (_native.Codec * len(arrays))(*[a.codec if a.codec is not None else _native.Codec(0, 0, 0, 0)
                                                 for a in arrays])
        rc = self.lib.secure_infer_h2d_reload_layers_async(0, len(arrays), srcs, dsts, n, counts, codecs,
                                                           1 if self.lookahead else 0, stream)
        if rc != 0:
            raise RuntimeError("secure_infer_h2d_reload_layers_async refused the request")
        return (srcs, dsts, counts, codecs)

    # ----------------------------------------------------------------- wait
    def wait_for_layer_load(self, name) -> None:
        """Every request being consumed has its KV for this layer before
        attention runs: with the host gate (the reference's behaviour) the
        layer's authentication is known on the host first; in both modes the
        current stream then waits on the layer's event, by which time any
        record that failed verification has been zeroed."""
        layer = self.names.index(name)
        stream = torch.cuda.current_stream(self.device)
        deadline = time.monotonic() + self.timeout
        gate = "authenticated" if self.host_gate else "submitted"
        for state in list(self.consuming.values()):
            with self.lock:
                while not state[gate][layer] and not state["error"]:
                    if not self.lock.wait(timeout=max(0.0, deadline - time.monotonic())):
                        if time.monotonic() >= deadline:
                            raise RuntimeError(f"layer {layer} not authenticated within {self.timeout} s")
                if state["error"]:
                    raise RuntimeError(state["error"])
                ready = state["ready_events"][layer]
                native = state.get("native", False)
            if native:
                if self.lib.secure_infer_layer_ready_wait(layer, ct.c_void_p(stream.cuda_stream)) != 0:
                    raise RuntimeError(f"layer {layer} has no reload to wait for")
            else:
                stream.wait_event(ready)
        if layer == len(self.names) - 1:
            for state in self.consuming.values():
                state["thread"].join(timeout=self.timeout)
                if state["thread"].is_alive():
                    raise RuntimeError("KV fetch thread timeout")
                if state["error"]:
                    raise RuntimeError(state["error"])
            self.consuming = {}

    # ------------------------------------------------------------- finished
    def get_finished(self) -> set:
        """Requests whose fetch completed since the last call; raises if any
        load failed."""
        with self.lock:
            for state in self.load_jobs.values():   # any failed load, finished or not (:412-416)
                if state["error"]:
                    raise RuntimeError(state["error"])
            done, self.newly_done = self.newly_done, set()
            for req_id in done:
                self.load_jobs.pop(req_id, None)
        return done

    def close(self) -> None:
        for state in list(self.load_jobs.values()):
            state["thread"].join(timeout=self.timeout)
        self.load_stream.synchronize()
