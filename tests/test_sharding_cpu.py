"""The N>1 host logic on CPU ranks (gloo, world size 2): bank sharding, per-rank output slices and the
optional all-gather reproduce the single-rank result column for column.  The oracle stands in for the
kernel (no GPU here); the CUDA path itself is covered by the gpu-marked tests."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

from tests import helpers as H


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def oracle_product(x, bank, name, drop):
    from oracle import reax_oracle as ro
    out = ro.gate_up_project(H.bits(x), H.bank_numpy(bank))
    return H.from_bits(out)


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from reax_engine_runtime_v3_b200.sharding import ShardedGateUp
        g = H.gen(5)
        x = H.activations(g, 9, 256)
        bank = H.int8_bank(g, 256, 512)
        op = ShardedGateUp(bank, rank, world, product=oracle_product)
        local = op.project(x)
        full = op.project(x, gather=True)
        shard = op.project(x, gather=True, layout="shard")
        q.put((rank, H.bits(local), H.bits(full), H.bits(shard)))
    finally:
        torch.distributed.destroy_process_group()


def test_two_rank_sharding_matches_single_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, local, full, shard = q.get(timeout=240)
        results[r] = (local, full, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = H.gen(5)
    x = H.activations(g, 9, 256)
    bank = H.int8_bank(g, 256, 512)
    whole = H.bits(oracle_product(x, bank, "", 0))
    h = 512 // world
    for r in range(world):
        local, full, shard = results[r]
        assert np.array_equal(local, whole[:, r * h:(r + 1) * h])
        assert np.array_equal(full, whole)
        assert np.array_equal(shard.reshape(world, 9, h).transpose(1, 0, 2).reshape(9, 512), whole)


def test_shard_rows_layout():
    from reax_engine_runtime_v3_b200.sharding import shard_rows
    rows, h = shard_rows(8, 1, 4)
    assert h == 2 and rows.tolist() == [2, 3, 10, 11]
