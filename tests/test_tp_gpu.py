"""Tensor-parallel engine on two GPUs (NCCL): every rank's output matches the
unsharded torch forward within the per-element budget.  Skipped with fewer
than two GPUs."""

import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    import os
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from oracle.model import ModelConfig, budget_usage, generate_case
        from tjkernels.model import Encoder, EncoderConfig, torch_forward
        from tjkernels.parallel import enable_tensor_parallel
        cfg = ModelConfig(2, 512, 1024, 16, 4096, 2, True)
        torch.manual_seed(0)
        enc = Encoder(EncoderConfig(2, 512, 1024, 16, 4096, 2, True)).to(dev).eval()
        x, mask = generate_case(cfg, 3, 0.5)
        x, mask = x.to(dev), mask.to(dev)
        with torch.no_grad():
            torch.backends.cuda.matmul.allow_tf32 = False
            want = torch_forward(enc, x, mask)
        enable_tensor_parallel(enc)
        with torch.inference_mode():
            got = enc(x, mask)
        out_q.put((rank, budget_usage(want[mask].cpu(), got[mask].cpu()),
                   bool((got[~mask] == 0).all())))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=300) for _ in range(2)]
    finally:
        # A worker that failed, or is still waiting on its peer, must not keep
        # holding its GPU after the test.
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    for rank, usage, zero in results:
        print(f"tensor parallel rank {rank}: budget usage {usage:.3f}")
        assert usage <= 1.0, (rank, usage)
        assert zero
