"""Host logic of the row-sharded encode with world_size 2 over gloo on CPU.

The per-rank encode is the CPU oracle here (the GPU path is exercised by the
GPU tests and bench.py over NCCL); what is tested is the sharding, the
padding of uneven shards, the all-gather and the reassembly — and that a
rank which fails before the collective makes the other rank error out
instead of hanging.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_codes_recon(x, cbs):
    from oracle import pyoracle as orc
    best, _, _, recon = orc.rvq_encode(_bits(x), _bits(cbs), threads=1)
    return torch.from_numpy(best), torch.from_numpy(orc.bf16_bits(recon).view(np.int16)).view(torch.bfloat16)


def _oracle_encode(x, cbs, sq, codes_out, recon_out):
    codes, recon = _oracle_codes_recon(x, cbs)
    codes_out.copy_(codes)
    recon_out.copy_(recon)


def _data(total, D, K, L):
    g = torch.Generator().manual_seed(7)
    x = torch.randn((total, D), generator=g).to(torch.bfloat16)
    cbs = (torch.randn((L, K, D), generator=g) * torch.tensor([0.5 ** l for l in range(L)]).view(L, 1, 1))
    return x, cbs.to(torch.bfloat16)


def _worker(rank, world, port, total, out_path, fail_rank):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from ncmorph_b200.sharded import shard_bounds, sharded_encode
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        x, cbs = _data(total, 16, 24, 3)
        start, stop, _ = shard_bounds(total, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        codes, recon = sharded_encode(x[start:stop], cbs, total, encode=_oracle_encode)
        if rank == 0:
            torch.save({"codes": codes, "recon": recon.view(torch.int16)}, out_path)
    except RuntimeError as e:
        with open(out_path + f".err{rank}", "w") as f:
            f.write(str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(total, fail_rank=-1):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.start_processes(_worker, args=(2, port, total, out, fail_rank), nprocs=2, join=True, start_method="spawn")
        errs = {r: open(out + f".err{r}").read() for r in range(2) if os.path.exists(out + f".err{r}")}
        res = torch.load(out) if os.path.exists(out) else None
    return res, errs


@pytest.mark.parametrize("total", [64, 101])
def test_sharded_encode_matches_single_process(total):
    res, errs = _run(total)
    assert not errs, errs
    x, cbs = _data(total, 16, 24, 3)
    codes, recon = _oracle_codes_recon(x, cbs)
    assert torch.equal(res["codes"], codes)
    assert torch.equal(res["recon"], recon.view(torch.int16))


def test_failed_rank_makes_peer_error_not_hang():
    res, errs = _run(64, fail_rank=1)
    assert res is None
    assert "injected failure" in errs.get(1, "")
    assert 0 in errs, "rank 0 should have seen the collective fail"


def test_shard_bounds_cover_rows_once():
    from ncmorph_b200.sharded import shard_bounds
    for total in (1, 7, 64, 1 << 20):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(total, world, r)[:2] for r in range(world)]
            covered = [i for a, b in spans for i in range(a, b)] if total < 100 else None
            if covered is not None:
                assert covered == list(range(total))
            assert spans[0][0] == 0 and spans[-1][1] == total


# ----------------------------------------------------- batch-sharded tokenizer
def _fake_tokenizer(x, w_in, codebooks, w_out, pool_factors, **kw):
    """Stands in for tokenizer_forward with the same shapes; every output of a
    batch item depends only on that item (as the real forward's do)."""
    b, T, Din = x.shape
    S, L, K, D = codebooks.shape
    xf = x.float()
    codes = []
    for f in pool_factors:
        pooled = xf.view(b, T // f, f, Din).mean(2).reshape(b * T // f, Din)
        codes.append(torch.stack([(pooled[:, l % Din] * 1000).round().to(torch.int32) + l for l in range(L)]))
    recon = xf[..., :D].to(torch.bfloat16)
    y = (xf * 2).to(torch.bfloat16)
    return codes, recon, y


def _tok_data(batch, T=16, Din=8, D=4, S=3, L=2, K=5):
    g = torch.Generator().manual_seed(11)
    x = torch.randn((batch, T, Din), generator=g).to(torch.bfloat16)
    cbs = torch.randn((S, L, K, D), generator=g).to(torch.bfloat16)
    return x, cbs, [4, 2, 1]


def _tok_worker(rank, world, port, batch, out_path, gather):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from ncmorph_b200.sharded import ShardedTokenizer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        x, cbs, pf = _tok_data(batch)
        tok = ShardedTokenizer(batch, x.shape[1], pf, forward=_fake_tokenizer, gather=gather)
        codes, recon, y = tok(x[tok.b0:tok.b1], None, cbs, None)
        torch.save({"codes": codes, "recon": recon.view(torch.int16), "y": y.view(torch.int16),
                    "items": tok.items, "b0": tok.b0, "b1": tok.b1}, out_path + f".{rank}")
    except Exception as e:  # noqa: BLE001
        with open(out_path + f".err{rank}", "w") as f:
            f.write(repr(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("world,batch,gather", [(2, 4, "all"), (2, 3, "all"), (3, 2, "all"), (2, 3, "codes"),
                                                (3, 2, "codes")])
def test_sharded_tokenizer_matches_single_process(world, batch, gather):
    """Whole batch items per rank (uneven, and a rank with none): every rank
    gets the codes of every scale in the batch order of one forward over the
    whole batch, and with gather="all" the reconstructions and outputs too
    (else its own items' ones)."""
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "tok")
        mp.start_processes(_tok_worker, args=(world, port, batch, out, gather), nprocs=world, join=True,
                           start_method="spawn")
        errs = {r: open(out + f".err{r}").read() for r in range(world) if os.path.exists(out + f".err{r}")}
        assert not errs, errs
        res = [torch.load(out + f".{r}") for r in range(world)]
    x, cbs, pf = _tok_data(batch)
    codes, recon, y = _fake_tokenizer(x, None, cbs, None, pf)
    assert sum(r["items"] for r in res) == batch
    for r in res:
        assert len(r["codes"]) == len(pf)
        for s in range(len(pf)):
            assert torch.equal(r["codes"][s], codes[s]), (s, r["codes"][s], codes[s])
        sl = slice(None) if gather == "all" else slice(r["b0"], r["b1"])
        assert torch.equal(r["recon"], recon[sl].view(torch.int16))
        assert torch.equal(r["y"], y[sl].view(torch.int16))
