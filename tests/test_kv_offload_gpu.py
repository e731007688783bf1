"""GPU tests of the codec transfer objects (EncodedStore, PackedTransfer,
PipelinedTransfer): packets bit-exact with the oracle encode, reloads
bit-exact with the oracle decode, stale slots refused, recovery callbacks."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import det_bytes
from oracle import codec_oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KEY = det_bytes("offload-key", 16)
SALT = det_bytes("offload-salt", 4)


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from secure_infer_b200 import kv_offload, native_layerwise
    s = native_layerwise.Session(0, KEY, SALT)
    yield kv_offload, native_layerwise
    s.close()


def u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def make_caches(layers, blocks, heads, seed):
    g = torch.Generator().manual_seed(seed)
    return [[torch.randn((blocks, 128, heads, 128), generator=g).to(torch.bfloat16).cuda() for _ in range(2)]
            for _ in range(layers)]


def expected_decode(packets, bits, kind, heads, n):
    qb, sb = 128 * heads * 128 * bits // 8, 128 * heads * 128 // 64 * 4
    out = np.zeros((n, 128, heads, 128), np.uint16)
    codec_oracle.decode_into(packets, out, np.arange(n), bits, kind, qb, sb)
    return out


def test_encoded_store_packets_versions_and_reload(mods):
    ko, nl = mods
    layers, heads, slots, mode = 3, 2, 6, "mixed"
    caches = make_caches(layers, 8, heads, 11)
    store = ko.EncodedStore(slots, layers, heads, mode)
    gpu_blocks, cpu_slots = [7, 1, 4, 2], [0, 3, 5, 1]
    store.submit("job-a", cpu_slots)
    for layer in range(layers):
        store.store_layer("job-a", layer, caches[layer], gpu_blocks)
    with pytest.raises(RuntimeError, match="stale"):
        store.get(0, 0, nl.layer_bits(mode, 0, layers), cpu_slots)   # not yet published
    assert store.finished() == ["job-a"]
    for layer in range(layers):
        bits = nl.layer_bits(mode, layer, layers)
        for kind in range(2):
            cpu, qb, sb = store.get(layer, kind, bits, cpu_slots)
            want, _, _ = codec_oracle.encode(u16(caches[layer][kind]), gpu_blocks, bits, kind, layer)
            assert np.array_equal(cpu.numpy()[cpu_slots], want), (layer, kind)
    # Reload through PackedTransfer into a fresh paged cache.
    dest = [[torch.zeros((9, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
            for _ in range(layers)]
    mapping = torch.tensor([[3, 8], [0, 2], [5, 0], [1, 6]])
    t = ko.PackedTransfer(store)
    for layer in range(layers):
        t.transfer((None, mapping), dest[layer])
        t.wait_for_layer_load(layer)
        bits = nl.layer_bits(mode, layer, layers)
        for kind in range(2):
            cpu, _, _ = store.get(layer, kind, bits, cpu_slots)
            exp = expected_decode(cpu.numpy()[mapping[:, 0].numpy()], bits, kind, heads, len(mapping))
            assert np.array_equal(u16(dest[layer][kind])[mapping[:, 1].numpy()], exp), (layer, kind)
    # A later store of slot 3 makes it stale until that store is published.
    store.submit("job-b", [3])
    with pytest.raises(RuntimeError, match="stale"):
        store.get(0, 0, nl.layer_bits(mode, 0, layers), [3])
    store.get(0, 0, nl.layer_bits(mode, 0, layers), [0, 5, 1])          # untouched slots stay valid
    for layer in range(layers):
        store.store_layer("job-b", layer, caches[layer], [6])
    store.wait(["job-b"])
    cpu, _, _ = store.get(0, 0, nl.layer_bits(mode, 0, layers), [3])
    want, _, _ = codec_oracle.encode(u16(caches[0][0]), [6], nl.layer_bits(mode, 0, layers), 0, 0)
    assert np.array_equal(cpu.numpy()[3], want[0])
    with pytest.raises(RuntimeError, match="No encoded cache"):
        store.get(layers + 5, 0, 8, [0])


def test_pipelined_transfer_callbacks_and_errors(mods):
    ko, nl = mods
    layers, heads, slots, mode = 4, 1, 4, "int8"
    caches = make_caches(layers, 4, heads, 23)
    store = ko.EncodedStore(slots, layers, heads, mode)
    store.submit(1, range(4))
    for layer in range(layers):
        store.store_layer(1, layer, caches[layer], range(4))
    store.finished()
    dest = [[torch.zeros((4, 128, heads, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
            for _ in range(layers)]
    mapping = torch.tensor([[2, 0], [0, 1], [3, 2], [1, 3]])
    ready, errors = [], []
    t = ko.PipelinedTransfer(store)
    t.start_request("req", mode, layers, lambda layer, ev, start: ready.append((layer, ev)), errors.append)
    for layer in range(layers):
        t.transfer((None, mapping), dest[layer])
    t.finish_request()
    assert [layer for layer, _ in ready] == list(range(layers)) and not errors
    consumer = torch.cuda.Stream()
    for layer, ev in ready:
        consumer.wait_event(ev)
    torch.cuda.synchronize()
    for layer in range(layers):
        for kind in range(2):
            cpu, _, _ = store.get(layer, kind, 8, range(4))
            exp = expected_decode(cpu.numpy()[mapping[:, 0].numpy()], 8, kind, heads, 4)
            assert np.array_equal(u16(dest[layer][kind])[mapping[:, 1].numpy()], exp)
    # An authentication failure reaches on_error and finish_request raises.
    t2 = ko.PipelinedTransfer(store)
    t2.wait_auth = lambda layer: -1 if layer == 1 else 0
    ready.clear()
    t2.start_request("req2", mode, layers, lambda layer, ev, start: ready.append(layer), errors.append)
    with pytest.raises(RuntimeError, match="authentication failed"):
        for layer in range(layers):
            t2.transfer((None, mapping), dest[layer])
        t2.finish_request()
    assert errors and "authentication failed" in errors[0] and ready == [0]
    for layer in range(layers):
        nl.NativeTransfer("none").lib.secure_infer_recovery_wait_layer_authentication(layer)
