"""Batch sharding across ranks (CPU, gloo, world size 2).

Sequences are independent in the encoder (row-wise GEMMs and LayerNorms,
attention within a sequence), so the multi-GPU forward shards the batch with
no collective: each rank runs its contiguous slice and the results
concatenate to the single-process forward.  Checked here with the CPU oracle
on two gloo ranks, plus the host-side shard arithmetic.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.model import ModelConfig, build_model, generate_case, oracle_forward


def test_shard_range_covers_batch():
    from tjkernels.parallel import shard_range
    for batch in (1, 7, 8, 64):
        for world in (1, 2, 3, 8):
            spans = [shard_range(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def test_balanced_shards_balance_causal_work():
    from tjkernels.parallel import balanced_shards
    lengths = [2048, 1024, 1500, 1100, 2000, 1300, 1800, 1024]
    shards = balanced_shards(lengths, 4)
    assert sorted(i for s in shards for i in s) == list(range(8))
    load = [sum(lengths[i] * (lengths[i] + 1) / 2 + lengths[i] for i in s) for s in shards]
    assert max(load) / min(load) < 1.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cfg, seed, pad, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tjkernels.parallel import shard_range
        torch.set_num_threads(1)
        model = build_model(cfg, 0)
        x, mask = generate_case(cfg, seed, pad)
        lo, hi = shard_range(cfg.batch_size, world, rank)
        local = oracle_forward(model, x[lo:hi], mask[lo:hi])
        # Shards differ by at most one sequence: gather padded to the largest.
        spans = [shard_range(cfg.batch_size, world, r) for r in range(world)]
        most = max(e - s for s, e in spans)
        padded = torch.zeros(most, cfg.seq_len, cfg.d_model)
        padded[: hi - lo] = local
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
        if rank == 0:
            torch.save(torch.cat([p[: e - s] for p, (s, e) in zip(parts, spans)]), out_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_batch_shard_equals_full_forward(tmp_path):
    cfg = ModelConfig(5, 48, 128, 2, 256, 2, True)
    out_path = str(tmp_path / "gathered.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), cfg, 7, 0.5, out_path), nprocs=2,
                       join=True, start_method="spawn")
    gathered = torch.load(out_path)
    model = build_model(cfg, 0)
    x, mask = generate_case(cfg, 7, 0.5)
    full = oracle_forward(model, x, mask)
    assert (gathered - full).abs().max().item() < 1e-5


def _leaver_main(rank, world, port, out_path):
    """Rank 1 leaves between steps without joining the barrier; rank 0 must
    get an error from the collective instead of waiting forever."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    dist.barrier()  # one healthy step
    if rank == 1:
        os._exit(0)  # dies with no collective in flight
    t0 = time.time()
    try:
        dist.barrier()
        outcome = "completed"
    except Exception as exc:  # gloo reports the lost peer or the timeout
        outcome = f"raised after {time.time() - t0:.1f}s: {type(exc).__name__}"
    with open(out_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_survivor_raises_when_a_rank_dies(tmp_path):
    out_path = str(tmp_path / "outcome.txt")
    mp.start_processes(_leaver_main, args=(2, _free_port(), out_path), nprocs=2, join=True,
                       start_method="spawn")
    with open(out_path) as f:
        outcome = f.read()
    assert outcome.startswith("raised"), outcome
    assert float(outcome.split()[2].rstrip("s:")) < 30.0


def test_balanced_equal_shards():
    from tjkernels.parallel import balanced_equal_shards
    import random
    rng = random.Random(7)
    for world in (1, 2, 4, 8):
        lengths = [rng.randint(1024, 2048) for _ in range(8 * world)]
        shards = balanced_equal_shards(lengths, world)
        assert sorted(i for sh in shards for i in sh) == list(range(len(lengths)))
        assert all(len(sh) == 8 for sh in shards)
        work = [sum(lengths[i] * (lengths[i] + 1) / 2 for i in sh) for sh in shards]
        assert max(work) / min(work) < 1.15
    with pytest.raises(ValueError):
        balanced_equal_shards([1, 2, 3], 2)


def _tp_worker(rank, world, port, out_q):
    import os
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.model import ModelConfig, generate_case
        from tjkernels.model import Encoder, EncoderConfig
        from tjkernels.parallel import tp_torch_forward
        cfg = ModelConfig(2, 40, 128, 4, 256, 2, True)
        torch.manual_seed(0)
        enc = Encoder(EncoderConfig(2, 40, 128, 4, 256, 2, True))
        x, mask = generate_case(cfg, 5, 0.5)
        with torch.no_grad():
            out = tp_torch_forward(enc, x, mask, rank, world)
        # A numpy copy travels by value; a tensor would travel through shared
        # memory that this process may remove by exiting before it is read.
        out_q.put((rank, out.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_math_matches_unsharded(world):
    """Column-parallel QKV / FFN-in, row-parallel out-proj / FFN-out with an
    all-reduce (gloo ranks on the CPU) give every rank the unsharded forward."""
    import torch.multiprocessing as mp
    from oracle.model import ModelConfig, generate_case
    from tjkernels.model import Encoder, EncoderConfig, torch_forward
    cfg = ModelConfig(2, 40, 128, 4, 256, 2, True)
    torch.manual_seed(0)
    enc = Encoder(EncoderConfig(2, 40, 128, 4, 256, 2, True))
    x, mask = generate_case(cfg, 5, 0.5)
    with torch.no_grad():
        want = torch_forward(enc, x, mask)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = {r: torch.from_numpy(a) for r, a in (q.get(timeout=180) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert (outs[r] - want).abs().max().item() < 1e-4
        assert bool((outs[r][~mask] == 0).all())


def test_tp_shard_shapes_and_errors():
    from tjkernels.model import Encoder, EncoderConfig
    from tjkernels.parallel import tp_shard
    torch.manual_seed(0)
    enc = Encoder(EncoderConfig(1, 8, 64, 4, 256, 1, True))
    w = tp_shard(enc.layers[0], 1, 4)
    assert w["wqkv"].shape == (48, 64) and w["wo"].shape == (64, 16)
    assert w["w1"].shape == (64, 64) and w["w2"].shape == (64, 64)
    assert torch.equal(w["wqkv"][:16], enc.layers[0].attention.q_proj.weight[16:32])
    with pytest.raises(ValueError):
        tp_shard(enc.layers[0], 0, 3)


def _peer_rank_main(rank, world, port, nccl_env, out_path):
    import sys
    from pathlib import Path
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if nccl_env:
        os.environ["BENCH_SG_NCCL"] = "1"
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
        import bench
        dev = torch.device("cpu")
        inputs = [torch.zeros(4) for _ in range(world)] if rank == 0 else []
        peers = bench.PeerBuffers(dist, rank, world, dev, 16, 2, inputs)
        # Every rank agrees, and the collectives after it still line up.
        flag = torch.tensor([1 if peers.ok else 0])
        dist.all_reduce(flag)
        torch.save({"ok": peers.ok, "sum": int(flag.item())}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nccl_env", [False, True])
def test_peer_buffers_fall_back_together(tmp_path, nccl_env):
    """The copy-engine scatter/gather set-up of bench.py on two gloo ranks
    without a GPU: it cannot map device memory, so every rank reports the
    NCCL fallback and all ranks still take the same collective steps."""
    port = _free_port()
    out = str(tmp_path / "peer")
    mp.spawn(_peer_rank_main, args=(2, port, nccl_env, out), nprocs=2, join=True)
    for r in range(2):
        got = torch.load(f"{out}.{r}")
        assert got["ok"] is False and got["sum"] == 0
