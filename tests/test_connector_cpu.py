"""Host logic of the worker-side reload connector (LayerwiseReloader) on the
CPU: the CUDA streams and events, the native library and the transfer object
are replaced by fakes, and failures are made on the host (an authentication
wait that reports -1, a transfer that raises, an authentication wait that
never returns), so the thread hand-offs, error propagation and timeouts are
tested without a GPU."""
from __future__ import annotations

import threading
import time
import types

import pytest

torch = pytest.importorskip("torch")

LAYERS = 4


class FakeEvent:
    def __init__(self, *a, **k):
        self.recorded = False

    def record(self, stream=None):
        self.recorded = True


class FakeStream:
    cuda_stream = 0

    def __init__(self, *a, **k):
        self.waited = []

    def wait_event(self, ev):
        self.waited.append(ev)

    def synchronize(self):
        pass


class FakeCuda:
    Event = FakeEvent
    Stream = FakeStream

    def __init__(self):
        self.current = FakeStream()

    def current_stream(self, device=None):
        return self.current

    def set_device(self, device):
        pass

    def stream(self, s):
        class Ctx:
            def __enter__(self_inner):
                return s

            def __exit__(self_inner, *a):
                return False
        return Ctx()


class FakeLib:
    """Authentication waits succeed, except `fail_layer` (reports -1 once
    `gate` is set) and `hang_layer` (returns only when `release` is set)."""

    def __init__(self, fail_layer=None, hang_layer=None):
        self.fail_layer, self.hang_layer = fail_layer, hang_layer
        self.release = threading.Event()
        self.gate = threading.Event()
        self.calls = []

    def secure_infer_recovery_set_job_id(self, job):
        pass

    def secure_infer_recovery_wait_layer_authentication(self, layer):
        self.calls.append(layer)
        if layer == self.hang_layer:
            self.release.wait(timeout=30)
        if layer == self.fail_layer:
            self.gate.wait(timeout=30)
            return -1
        return 0

    def secure_infer_retire_transfer_prefetches(self):
        pass


class FakeTransfer:
    raise_on_layer = None
    gate = threading.Event()

    def __init__(self, mode, layers=1, heads=None):
        self.layer = 0

    def prepare_layer(self, payload, heads, layer=None):
        return True

    def single_layer_kv_transfer(self, payload, destination, stream=None):
        if self.layer == FakeTransfer.raise_on_layer:
            FakeTransfer.gate.wait(timeout=30)
            raise ValueError(f"transfer of layer {self.layer} refused")

    def layer_arrays(self, payload, destination, layer):
        return layer

    def prepare_arrays(self, arrays):
        return True

    def reload_arrays(self, layer, stream):
        self.layer = layer
        self.single_layer_kv_transfer(None, None, stream)


@pytest.fixture
def make(monkeypatch):
    from secure_infer_b200 import connector

    def build(lib, timeout=5.0, raise_on_layer=None, host_gate=True):
        fake_torch = types.SimpleNamespace(cuda=FakeCuda(), from_numpy=torch.from_numpy)
        monkeypatch.setattr(connector, "torch", fake_torch)
        monkeypatch.setattr(connector._native, "lib", lambda: lib)
        FakeTransfer.raise_on_layer = raise_on_layer
        FakeTransfer.gate = threading.Event()
        monkeypatch.setattr(connector, "NativeTransfer", FakeTransfer)
        caches = [[torch.zeros((8, 4, 1, 4)) for _ in range(2)] for _ in range(LAYERS)]
        cpu = [[torch.zeros((8, 4, 1, 4)) for _ in range(2)] for _ in range(LAYERS)]
        names = [f"layers.{i}" for i in range(LAYERS)]
        return (connector.LayerwiseReloader(names, caches, cpu, mode="none", timeout=timeout, host_gate=host_gate),
                names, fake_torch)
    return build


def test_all_layers_released_in_order(make):
    lib = FakeLib()
    r, names, ft = make(lib)
    r.start_load("a", [1, 2], [3, 4])
    for name in names:
        r.wait_for_layer_load(name)
    assert lib.calls == list(range(LAYERS))
    assert len(ft.cuda.current.waited) == LAYERS          # one device wait per layer
    assert r.get_finished() == {"a"}


def test_authentication_failure_reaches_its_layer(make):
    """Layers authenticated before the failure are released; once a layer
    fails, every wait of the request raises the reference's message (like its
    `assert not state['error']`), and the failure sticks for later loads."""
    lib = FakeLib(fail_layer=2)
    r, names, _ = make(lib)
    r.start_load("a", [0], [0])
    r.wait_for_layer_load(names[0])
    r.wait_for_layer_load(names[1])
    lib.gate.set()
    with pytest.raises(RuntimeError, match="Packed KV authentication failed"):
        r.wait_for_layer_load(names[2])
    with pytest.raises(RuntimeError, match="Packed KV authentication failed"):
        r.get_finished()
    r.load_jobs["a"]["thread"].join(timeout=10)
    r.load_jobs.clear()
    r.consuming = {}
    r.start_load("b", [0], [0])
    with pytest.raises(RuntimeError, match="Packed KV authentication failed"):
        r.wait_for_layer_load(names[0])


def test_transfer_exception_is_reported_first(make):
    r, names, _ = make(FakeLib(), raise_on_layer=1)
    r.start_load("a", [0], [0])
    r.wait_for_layer_load(names[0])
    FakeTransfer.gate.set()
    with pytest.raises(RuntimeError, match="transfer of layer 1 refused"):
        r.wait_for_layer_load(names[1])


def test_stalled_authentication_times_out(make):
    """An authentication wait that does not return within the connector's
    timeout ends the layer wait with an error instead of blocking forever."""
    lib = FakeLib(hang_layer=1)
    r, names, _ = make(lib, timeout=0.5)
    r.start_load("a", [0], [0])
    r.wait_for_layer_load(names[0])
    t0 = time.monotonic()
    with pytest.raises(RuntimeError, match="not authenticated within|authentication observer timeout"):
        r.wait_for_layer_load(names[1])
    assert time.monotonic() - t0 < 10
    lib.release.set()
    r.load_jobs["a"]["thread"].join(timeout=10)


def test_block_indices_checked(make):
    r, _, _ = make(FakeLib())
    with pytest.raises(ValueError):
        r.start_load("a", [8], [0])
    with pytest.raises(ValueError):
        r.start_load("a", [0, 1], [0])


def test_device_gate_releases_layers_before_host_authentication(make):
    """host_gate=False: a layer is released to the compute stream once it is
    submitted, while its authentication is still pending on the host; the
    last layer still joins the request and reports its outcome."""
    lib = FakeLib(hang_layer=1)
    r, names, ft = make(lib, host_gate=False)
    r.start_load("a", [0], [0])
    t0 = time.monotonic()
    for name in names[:-1]:
        r.wait_for_layer_load(name)              # layer 1's authentication is still pending
    assert time.monotonic() - t0 < 3.0
    assert len(ft.cuda.current.waited) == LAYERS - 1
    lib.release.set()
    r.wait_for_layer_load(names[-1])
    assert r.get_finished() == {"a"}
