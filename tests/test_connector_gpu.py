"""GPU test of the worker-side reload connector (LayerwiseReloader), the CUDA
form of RuntimeWorker in secure_infer/reuse/connector.py: per-layer reloads on
a load stream with lookahead, authentication observed per layer, and a
compute stream that only waits on device events before "attention" reads the
layer."""
from __future__ import annotations

import pytest

from conftest import det_bytes

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("connector-key", 16)
SALT = det_bytes("connector-salt", 4)
LAYERS, HEADS, POOL, CACHE = 4, 2, 12, 16


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import native_layerwise as nl
    s = nl.Session(0, KEY, SALT)
    g = torch.Generator().manual_seed(7)
    cpu = [[torch.randn((POOL, 128, HEADS, 128), generator=g).to(torch.bfloat16).pin_memory() for _ in range(2)]
           for _ in range(LAYERS)]
    for layer in range(LAYERS):
        for k in range(2):
            nl.register_host_range(cpu[layer][k], layer, k)
    yield nl, cpu
    s.close()


def make_reloader(cpu, mode="none", native_loop=False, host_gate=True):
    from secure_infer_b200.connector import LayerwiseReloader
    caches = [[torch.zeros((CACHE, 128, HEADS, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
              for _ in range(LAYERS)]
    names = [f"model.layers.{i}.self_attn" for i in range(LAYERS)]
    return (LayerwiseReloader(names, caches, cpu, mode=mode, native_loop=native_loop, host_gate=host_gate), caches,
            names)


def run_model(reloader, names, caches, dest):
    """Per layer: wait for the layer, then read it on the compute stream."""
    sums = []
    for layer, name in enumerate(names):
        reloader.wait_for_layer_load(name)
        sums.append(torch.stack([caches[layer][k][dest].float().sum() for k in range(2)]))
    torch.cuda.synchronize()
    return torch.stack(sums).cpu()


def expected(cpu, src):
    return torch.stack([torch.stack([cpu[layer][k][src].float().sum() for k in range(2)])
                        for layer in range(LAYERS)])


@pytest.mark.parametrize("native_loop,host_gate", [(False, True), (True, True), (False, False), (True, False)])
def test_two_requests_reload_all_layers(env, native_loop, host_gate):
    """The layer loop in the connector's fetch thread or on the library's
    thread (secure_infer_h2d_reload_layers_async), attention gated after host
    authentication or on the device alone: the same blocks land either way."""
    nl, cpu = env
    reloader, caches, names = make_reloader(cpu, native_loop=native_loop, host_gate=host_gate)
    for req, (src, dst) in enumerate([([3, 0, 7, 5], [10, 2, 4, 9]), ([11, 1], [0, 15])]):
        before = nl.prefetch_stats()
        reloader.start_load(f"req-{req}", src, dst)
        got = run_model(reloader, names, caches, dst)
        # Device and host sums differ only in summation order (fp32 tolerance);
        # the blocks themselves are compared bit for bit below.
        assert torch.allclose(got, expected(cpu, src), rtol=1e-5, atol=1e-3)
        for layer in range(LAYERS):
            for k in range(2):
                assert torch.equal(caches[layer][k][dst].cpu(), cpu[layer][k][src])
        assert reloader.get_finished() == {f"req-{req}"}
        assert nl.prefetch_stats()["ready"] - before["ready"] == (LAYERS - 1) * 2 * len(src)
    reloader.close()


def test_tampered_record_retried(env):
    nl, cpu = env
    reloader, caches, names = make_reloader(cpu)
    before = nl.auth_stats()
    nl._native.lib().secure_infer_arm_tamper(1, 3, 0)
    src, dst = [2, 4, 6], [1, 3, 5]
    reloader.start_load("tamper", src, dst)
    got = run_model(reloader, names, caches, dst)
    assert torch.allclose(got, expected(cpu, src), rtol=1e-5, atol=1e-3)
    for layer in range(LAYERS):
        for k in range(2):
            assert torch.equal(caches[layer][k][dst].cpu(), cpu[layer][k][src])
    after = nl.auth_stats()
    assert after["rejected"] - before["rejected"] == 1 and after["retried"] - before["retried"] == 1
    assert reloader.get_finished() == {"tamper"}
    reloader.close()


def test_fetch_failure_reaches_layer_wait_and_sticks(env):
    """A failure inside the fetch thread (here: host pools that are not codec
    packets) reaches wait_for_layer_load as RuntimeError, and later loads are
    refused, like the reference's sticky load_failure."""
    nl, cpu = env
    reloader, caches, names = make_reloader(cpu, mode="int8")
    reloader.start_load("bad", [0, 1], [0, 1])
    with pytest.raises(RuntimeError, match="packet width"):
        reloader.wait_for_layer_load(names[0])
    with pytest.raises(RuntimeError):
        reloader.get_finished()
    reloader.load_jobs["bad"]["thread"].join(timeout=60)
    reloader.load_jobs.clear()
    reloader.consuming = {}
    reloader.start_load("after", [0], [0])
    with pytest.raises(RuntimeError, match="packet width"):
        reloader.wait_for_layer_load(names[0])
    with pytest.raises(ValueError):
        reloader.start_load("range", [POOL], [0])
    reloader.close()
