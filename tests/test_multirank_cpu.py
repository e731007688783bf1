"""World-size-2 gloo test of the multi-rank host logic (no GPU).

Each rank (one TP shard) runs its own host-only session with the key and salt
bench.py gives it, encrypts records for its own KV heads, and the ranks
exchange what they produced: a rank's records authenticate under its own
session and under no other, each rank process numbers its tickets from 1,
and the job time is the maximum over ranks.
"""
from __future__ import annotations

import ctypes as ct
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

COUNT, N = 4096, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import gcm as orc
    from secure_infer_b200 import _native

    dist.init_process_group("gloo", rank=rank, world_size=world)
    lib = _native.lib()
    key, salt = bench.rank_session_material(rank)
    assert lib.secure_infer_session_init(-1, (ct.c_uint8 * 16)(*key), (ct.c_uint8 * 4)(*salt)) == 0
    kv = np.frombuffer(os.urandom(COUNT * N), np.uint8).reshape(N, COUNT).copy()
    lib.secure_infer_register_host_range_ex(kv.ctypes.data, kv.nbytes, 3, rank % 2, COUNT)
    stride = lib.secure_infer_record_bytes(COUNT)
    recs = np.zeros((N, stride), np.uint8)
    tickets = (ct.c_uint64 * N)()
    srcs = (ct.c_void_p * N)(*[kv.ctypes.data + i * COUNT for i in range(N)])
    assert lib.secure_infer_h2d_encrypt_records(srcs, COUNT, N, recs.ctypes.data, stride, tickets) == 0
    assert list(tickets) == list(range(1, N + 1))      # each rank process has its own ticket counter

    mine = torch.from_numpy(recs.copy())
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    aligned = orc.record_aligned_bytes(COUNT)
    for other in range(world):
        okey, osalt = bench.rank_session_material(other)
        for src_rank in range(world):
            rec = gathered[src_rank].numpy()[0]
            iv = orc.derive_transfer_iv(osalt, 1)
            plain, ok = orc.host_decrypt_verify(okey, iv, rec[aligned + 32:].tobytes(), rec[:COUNT].tobytes(),
                                                rec[aligned:aligned + 16].tobytes())
            assert ok == (1 if other == src_rank else 0), (rank, other, src_rank)
            if other == src_rank == rank:
                assert plain == kv[0].tobytes()

    t = bench.max_over_ranks(1.5 + rank, dist, device="cpu")
    assert t == 1.5 + (world - 1)
    lib.secure_infer_session_shutdown()
    dist.destroy_process_group()
    open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")


def test_two_rank_sessions_are_independent(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]


def _pool_info_child(local_rank: int, local_world: int):
    import sys
    os.environ.update(LOCAL_RANK=str(local_rank), LOCAL_WORLD_SIZE=str(local_world))
    os.environ.pop("SECURE_INFER_CRYPTO_THREADS", None)
    os.environ.pop("SECURE_INFER_PIN_THREADS", None)
    sys.path.insert(0, str(ROOT))
    from secure_infer_b200 import _native
    info = _native.host_pool_info()
    return info, sorted(os.sched_getaffinity(0))


def test_ranks_sharing_a_host_split_its_cpus():
    """Ranks on one host (LOCAL_WORLD_SIZE > 1) size and pin their OpenSSL
    pools to disjoint equal slices of the CPUs instead of each starting a pool
    as large as the host; a lone rank uses every CPU, unpinned."""
    import multiprocessing as mpc
    ctx = mpc.get_context("spawn")
    local_world = 2
    with ctx.Pool(1) as p:
        alone, cpus = p.apply(_pool_info_child, (0, 1))
    assert alone["cpus"] == cpus and not alone["pinned"]
    assert alone["threads"] == min(len(cpus) - 1, 31)
    slices = []
    for r in range(local_world):
        with ctx.Pool(1) as p:
            info, _ = p.apply(_pool_info_child, (r, local_world))
        share = max(1, len(cpus) // local_world)
        assert len(info["cpus"]) == share and info["pinned"]
        assert info["threads"] == share - 1
        slices.append(set(info["cpus"]))
    assert not (slices[0] & slices[1]) or len(cpus) < local_world
