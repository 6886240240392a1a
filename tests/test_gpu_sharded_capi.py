"""Row-sharded encode through the C ABI's own NCCL communicator
(ncm_ctx_comm_init + ncm_rvq_encode_sharded) on 2 GPUs: every rank's
gathered codes and reconstructions equal a single-GPU encode of all rows.
Skipped on a box with fewer than 2 GPUs."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, uid, nranks, n_local, out_dir):
    import numpy as np  # noqa: F401
    from ncmorph_b200 import sharded, vq
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    N, D, K, L = n_local * nranks, 256, 1024, 3
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((N, D), generator=g, device=dev).to(torch.bfloat16)
    cbs = torch.randn((L, K, D), generator=g, device=dev).to(torch.bfloat16)
    sharded.comm_init(dev, uid, rank, nranks)
    codes, recon = sharded.rvq_encode_sharded(x[rank * n_local:(rank + 1) * n_local].contiguous(), cbs, nranks)
    ref_codes, ref_recon, _ = vq.rvq_encode(x, cbs)
    torch.cuda.synchronize(dev)
    ok = torch.equal(codes, ref_codes) and torch.equal(recon.view(torch.int16), ref_recon.view(torch.int16))
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")


def test_sharded_encode_capi_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from ncmorph_b200 import sharded
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = sharded.comm_unique_id()
    ctx = mp.start_processes(_worker, args=(uid, 2, 4096, str(tmp_path)), nprocs=2, join=False, start_method="spawn")
    import time
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("sharded encode did not finish within 240 s")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"


def _worker_overlap(rank, nranks, port, total, out_dir, transport):
    import datetime

    import torch.distributed as dist
    from ncmorph_b200 import sharded, vq
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=nranks, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        N, D, K, L = total, 256, 1024, 3
        g = torch.Generator(device=dev).manual_seed(6)
        xs = [torch.randn((N, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
        cbs = torch.randn((L, K, D), generator=g, device=dev).to(torch.bfloat16)
        enc = sharded.ShardedEncoder(cbs, N, overlap=True, transport=transport)
        ok = True
        # three calls: both buffer sets, the first one reused by the third call
        outs = [enc(x[enc.start:enc.stop].contiguous()) for x in xs]
        enc.wait()
        torch.cuda.synchronize(dev)
        for x, (codes, recon) in zip(xs[1:], outs[1:]):  # the first call's buffers were reused by the third
            ref_codes, ref_recon, _ = vq.rvq_encode(x, cbs)
            ok = ok and torch.equal(codes, ref_codes) and torch.equal(recon.view(torch.int16),
                                                                     ref_recon.view(torch.int16))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
        enc.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport,total", [("nccl", 8192), ("peer", 8192), ("peer", 8092)])
def test_sharded_encoder_overlapped_gathers_two_gpus(tmp_path, transport, total):
    """ShardedEncoder(overlap=True): the all-gathers (NCCL kernels, or
    copy-engine pushes into the peers' IPC-mapped buffers) run on a second
    stream while the next call encodes; results equal a single-GPU encode,
    with even shards and with a short last shard."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import time

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.start_processes(_worker_overlap, args=(2, port, total, str(tmp_path), transport), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("overlapped sharded encode did not finish within 240 s")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"


def _worker_tokenizer(rank, nranks, port, batch, out_dir):
    import datetime

    import torch.distributed as dist
    from ncmorph_b200 import sharded, vq
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=nranks, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        T, Din, D, K, S, L, pf = 512, 512, 256, 512, 3, 3, [4, 2, 1]
        g = torch.Generator(device=dev).manual_seed(8)
        x = torch.randn((batch, T, Din), generator=g, device=dev).to(torch.bfloat16)
        w_in = (torch.randn((D, Din), generator=g, device=dev) * 0.05).to(torch.bfloat16)
        w_out = (torch.randn((Din, D), generator=g, device=dev) * 0.05).to(torch.bfloat16)
        cbs = (torch.randn((S, L, K, D), generator=g, device=dev)).to(torch.bfloat16)
        tok = sharded.ShardedTokenizer(batch, T, pf, gather="all")
        codes, recon, y = tok(x[tok.b0:tok.b1].contiguous(), w_in, cbs, w_out)
        # reference: each rank's items through one single-GPU forward, in batch order
        refs = []
        for r in range(nranks):
            b0, b1, _ = sharded.shard_bounds(batch, nranks, r)
            if b1 > b0:
                refs.append(vq.tokenizer_forward(x[b0:b1].contiguous(), w_in, cbs, w_out, pf))
        torch.cuda.synchronize(dev)
        ok = all(torch.equal(codes[s], torch.cat([c[s] for c, _, _ in refs], 1)) for s in range(S))
        ok = ok and torch.equal(recon.view(torch.int16), torch.cat([rc for _, rc, _ in refs]).view(torch.int16))
        ok = ok and torch.equal(y.view(torch.int16), torch.cat([yy for _, _, yy in refs]).view(torch.int16))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [4, 3])
def test_sharded_tokenizer_two_gpus(tmp_path, batch):
    """ShardedTokenizer: whole batch items per GPU (even, and 2 + 1), every
    rank's gathered codes, reconstructions and outputs equal the per-item
    single-GPU forwards in batch order, bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import time

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.start_processes(_worker_tokenizer, args=(2, port, batch, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("sharded tokenizer did not finish within 240 s")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
