"""Row-sharded gate/up and vocab matvecs across GPUs (NCCL all-gather).

Runs as one process per GPU (spawned here); skipped with fewer than 2 GPUs.
Rank 0 checks the gathered outputs against the unsharded oracle."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, kind, rows, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = False
    try:
        import oracle
        from mojo_llm_lab_b200 import fixtures as fx
        from mojo_llm_lab_b200 import ops
        from mojo_llm_lab_b200.shard import RowShard, all_gather_rows, assemble
        gen = fx.seeded_q6k_matrix if kind == "q6k" else fx.seeded_q4k_matrix
        row_bytes = k // 256 * (210 if kind == "q6k" else 144)
        host = [gen(rows, k, seed=3 + m) for m in range(1 if kind == "q6k" else 2)]
        x = fx.seeded_activation(k, seed=9)
        act = ops.quantize_q8_1(torch.from_numpy(x).cuda())
        shard = RowShard(rows, world, rank)
        mine = [shard.slice_weights(torch.from_numpy(w), row_bytes).cuda() for w in host]
        if kind == "q6k":
            local = ops.q6_k_q8_1_matvec(mine[0], act).view(1, -1)
        else:
            local = torch.stack(ops.q4k_gate_up(mine[0], mine[1], act))
        full = assemble(all_gather_rows(local, shard), shard).cpu().numpy().astype(np.float64)
        if rank == 0:
            a = oracle.quantize_q8_1(x)
            ref = [oracle.q6k_matvec(host[0], a, rows, k)] if kind == "q6k" else \
                list(oracle.q4k_gate_up(host[0], host[1], a, rows, k))
            ref = np.stack(ref)
            ok = bool(np.all(np.abs(full - ref) <= 1e-5 + 1e-5 * np.abs(ref)))
            q.put(ok)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,rows", [("gate_up", 9728), ("q6k", 151936)])
def test_sharded_over_all_gpus(kind, rows):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, rows, 2560, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    assert q.get(timeout=10) is True


def _spawn(target, world, *args):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes


def _gather_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from mojo_llm_lab_b200 import decode as D
        from mojo_llm_lab_b200 import ops
        from mojo_llm_lab_b200._lib import check, lib
        cfg = D.DecodeConfig(layers=1, vocab=4096, context=8, new_tokens=2)
        w = D.generate_weights(cfg, "cuda", world=world, rank=rank)
        k, v = D.generate_kv_cache(cfg, "cuda")
        dec = D.Decoder(w, k, v, group=dist.group.WORLD)
        assert dec.peer is not None, "symmetric memory unavailable"
        per = w.ffn_shard.per_rank
        results = []
        for it in range(4):  # alternate halves, several gathers
            g = torch.Generator(device="cuda")
            g.manual_seed(100 + it)
            full = torch.randn(cfg.ffn, generator=g, device="cuda") * (it + 1)
            dec.b.prod.copy_(full[rank * per:(rank + 1) * per])
            addr = dec._gather_prod(torch.cuda.current_stream().cuda_stream, 0, layer=it)
            torch.cuda.synchronize()
            got = torch.empty(cfg.ffn // 32 * 36, dtype=torch.uint8, device="cuda")
            got.copy_(dec.peer["buf"][addr - dec.peer["buf"].data_ptr():][:got.numel()])
            results.append(bool(torch.equal(got, ops.quantize_q8_1(full))))
        assert ops.device_error() == 0
        if rank == 0:
            torch.save(results, out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allgather_matches_local_quantisation(tmp_path):
    """Every rank's gathered Q8_1 equals the quantisation of the full vector, gather after gather."""
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    out = tmp_path / "gather.pt"
    _spawn(_gather_worker, world, out)
    assert torch.load(out) == [True] * 4


def _decode_worker(rank, world, port, out, gather="peer", gather_tail=True):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from mojo_llm_lab_b200 import decode as D
        cfg = D.DecodeConfig(layers=2, vocab=4096, context=300, new_tokens=6)
        w = D.generate_weights(cfg, "cuda", world=world, rank=rank)
        k, v = D.generate_kv_cache(cfg, "cuda")
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            dec = D.Decoder(w, k, v, group=dist.group.WORLD, gather=gather, gather_tail=gather_tail)
            assert (dec.peer is not None) == (gather == "peer")
            assert dec.gather_tail == (gather == "peer" and gather_tail)
            dec.reset(17)
            dec.capture()
            tokens = dec.generate(17, 5)
            logits = torch.empty(w.vocab_shard.per_rank * world, device="cuda")
            dist.all_gather_into_tensor(logits, dec.b.logits)
            s.synchronize()
            dec.graph = None
        if rank == 0:
            torch.save({"tokens": tokens, "logits": logits[:cfg.vocab].cpu()}, out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("gather,gather_tail", [("peer", True), ("peer", False), ("nccl", True)])
def test_sharded_decode_matches_single_gpu(tmp_path, gather, gather_tail):
    """gate/up + vocab row-sharded over the GPUs: the same tokens and logits as one GPU."""
    import torch
    from mojo_llm_lab_b200 import decode as D
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    out = tmp_path / "decode.pt"
    _spawn(_decode_worker, world, out, gather, gather_tail)
    got = torch.load(out)
    cfg = D.DecodeConfig(layers=2, vocab=4096, context=300, new_tokens=6)
    w = D.generate_weights(cfg, "cuda")
    k, v = D.generate_kv_cache(cfg, "cuda")
    dec = D.Decoder(w, k, v)
    tokens = dec.generate(17, 5)
    assert got["tokens"] == tokens
    assert torch.equal(got["logits"], dec.b.logits.cpu())
