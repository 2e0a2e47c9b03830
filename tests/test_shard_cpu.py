"""Host logic of the row-sharded matvecs on CPU ranks (gloo, world size 2).

Each rank computes its block of rows with the oracle (the GPU kernel's job on
a B200) and the blocks are all-gathered exactly as the NCCL path does; rank 0
checks the assembled vector against the unsharded oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mojo_llm_lab_b200 import fixtures as fx
from mojo_llm_lab_b200.shard import RowShard, all_gather_rows, assemble


@pytest.mark.parametrize("rows,world", [(9728, 2), (9728, 8), (151936, 8), (70, 4), (5, 8), (1, 2)])
def test_row_ranges_cover_every_row_once(rows, world):
    seen = []
    for r in range(world):
        s = RowShard(rows, world, r)
        assert s.per_rank * world >= rows
        seen.extend(range(s.start, s.stop))
    assert seen == list(range(rows))


def test_assemble_rank_major():
    shard = RowShard(10, 4, 0)  # per_rank 3, padded to 12
    gathered = torch.arange(4 * 2 * 3, dtype=torch.float32).view(4, 2, 3)
    full = assemble(gathered, shard)
    assert full.shape == (2, 10)
    assert full[0].tolist() == [0, 1, 2, 6, 7, 8, 12, 13, 14, 18]
    assert full[1].tolist() == [3, 4, 5, 9, 10, 11, 15, 16, 17, 21]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, kind, rows, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        gen = fx.seeded_q6k_matrix if kind == "q6k" else fx.seeded_q4k_matrix
        row_bytes = k // 256 * (210 if kind == "q6k" else 144)
        mats = [torch.from_numpy(gen(rows, k, seed=3 + m)) for m in range(1 if kind == "q6k" else 2)]
        act = oracle.quantize_q8_1(fx.seeded_activation(k, seed=9))
        shard = RowShard(rows, world, rank)
        mine = [shard.slice_weights(w, row_bytes).numpy() for w in mats]
        if kind == "q6k":
            local = [oracle.q6k_matvec(mine[0], act, shard.per_rank, k)]
        else:
            local = list(oracle.q4k_gate_up(mine[0], mine[1], act, shard.per_rank, k))
        local_t = torch.from_numpy(np.stack(local).astype(np.float64))
        full = assemble(all_gather_rows(local_t, shard), shard).numpy()
        if rank == 0:
            if kind == "q6k":
                ref = [oracle.q6k_matvec(mats[0].numpy(), act, rows, k)]
            else:
                ref = list(oracle.q4k_gate_up(mats[0].numpy(), mats[1].numpy(), act, rows, k))
            q.put(bool(np.array_equal(full, np.stack(ref))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,rows,world", [("gate_up", 300, 2), ("q6k", 257, 2), ("gate_up", 64, 4)])
def test_sharded_matvec_matches_unsharded(kind, rows, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, rows, 512, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=10) is True
