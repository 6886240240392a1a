"""Row-sharded RVQ encode: one process per GPU, codebooks replicated, codes
and reconstructions all-gathered over the process group (NCCL over NVLink on
a B200 node).

Token rows are independent at every RVQ step (research/reference/
vq_forward_semantics.md:59-82), so rank r encodes the contiguous block of
rows it owns and the only exchange is the all-gather of the int32 codes and
the bf16 reconstructions that the north star names. Shards have equal
padded length so that one all_gather_into_tensor per tensor suffices; padding
rows are never encoded and are trimmed after the gather.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_bounds(total_rows: int, world: int, rank: int) -> tuple[int, int, int]:
    """(start, stop, padded_len) of rank's contiguous row block."""
    if total_rows <= 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("bad sharding arguments")
    n = -(-total_rows // world)
    start = min(rank * n, total_rows)
    stop = min(start + n, total_rows)
    return start, stop, n


def _device_encode(x, codebooks, sqnorms, codes_out, recon_out):
    from . import vq
    vq.rvq_encode(x, codebooks, sqnorms, codes=codes_out, recon=recon_out)


class ShardedEncoder:
    """Encodes this rank's rows and all-gathers codes and reconstructions.

    `encode(x, codebooks, sqnorms, codes_out, recon_out)` fills the outputs
    ([L, n] int32 and [n, D]); it defaults to the tcgen05 path
    (ncmorph_b200.vq.rvq_encode). Buffers are allocated once; the tensors a
    call returns are views of them, valid until the next call.

    overlap=True streams batches: the all-gathers of a call run on a second
    stream while the next call already encodes (two buffer sets, so results
    stay valid until the call after next). Call `wait()` before the current
    stream reads a call's results; a device-wide synchronize also covers them.
    A call must be made after the caller's reads of the results of the call
    before last (on any stream) are ordered before the current stream.

    transport: "nccl" gathers with all_gather_into_tensor (NCCL kernels);
    "peer" pushes this rank's codes and reconstructions straight into every
    other rank's output buffers with copy-engine copies over CUDA IPC
    mappings (ncm_ipc_* / ncm_copy*_async), so the exchange takes no SMs
    from the encode it overlaps. Each peer exchange is bracketed by two
    one-element all-reduces on the group (every rank has finished encoding
    this call, so its buffers are free; every rank's copies have landed).
    The peer transport needs every rank on one node and overlap=True.
    """

    def __init__(self, codebooks: torch.Tensor, total_rows: int, x_dtype: torch.dtype = torch.bfloat16,
                 sqnorms: torch.Tensor | None = None, group=None, encode: Callable | None = None,
                 overlap: bool = False, transport: str = "nccl"):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.codebooks = codebooks
        self.sqnorms = sqnorms
        self.total = total_rows
        self.encode = encode or _device_encode
        self.start, self.stop, self.n = shard_bounds(total_rows, self.world, self.rank)
        L, D = codebooks.shape[0], codebooks.shape[-1]
        dev = codebooks.device
        self.L = L
        self.overlap = overlap
        sets = 2 if overlap else 1
        self.codes_pad = [torch.zeros((L, self.n), dtype=torch.int32, device=dev) for _ in range(sets)]
        self.recon_pad = [torch.zeros((self.n, D), dtype=x_dtype, device=dev) for _ in range(sets)]
        # outputs concatenated along dim 0 (the layout every backend accepts)
        self.codes_all = [torch.empty((self.world * L, self.n), dtype=torch.int32, device=dev) for _ in range(sets)]
        self.recon_all = [torch.empty((self.world * self.n, D), dtype=x_dtype, device=dev) for _ in range(sets)]
        self.codes_out = [torch.empty((L, self.world * self.n), dtype=torch.int32, device=dev) for _ in range(sets)]
        self.calls = 0
        if overlap:
            self.comm = torch.cuda.Stream(device=dev)
            self.encoded = [torch.cuda.Event() for _ in range(sets)]
            self.gathered = [torch.cuda.Event() for _ in range(sets)]
            self.used = [False] * sets
        if transport not in ("nccl", "peer"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.peers = None
        if transport == "peer" and self.world > 1:
            if not overlap:
                raise ValueError("the peer transport streams batches: use overlap=True")
            self._setup_peers()

    # ------------------------------------------------------------ peer transport
    def _setup_peers(self) -> None:
        """Exchanges the IPC handles of every rank's output buffers and maps
        the peers' ones: peers[b][r] = (codes_out base, recon_all base) of rank
        r's buffer set b, as addresses in this process."""
        import ctypes

        from . import _lib
        lib = _lib.load()
        mine = []
        for b in range(len(self.codes_out)):
            for t in (self.codes_out[b], self.recon_all[b]):
                h = _lib.IpcHandle()
                _lib.check(lib.ncm_ipc_export(ctypes.c_void_p(t.data_ptr()), t.numel() * t.element_size(),
                                              ctypes.byref(h)))
                mine.append(bytes(h))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.group)
        self.peers = []
        self._opened = []
        for b in range(len(self.codes_out)):
            row = []
            for r in range(self.world):
                if r == self.rank:
                    row.append((self.codes_out[b].data_ptr(), self.recon_all[b].data_ptr()))
                    continue
                ptrs = []
                for k in range(2):
                    h = _lib.IpcHandle.from_buffer_copy(everyone[r][2 * b + k])
                    p = ctypes.c_void_p()
                    _lib.check(lib.ncm_ipc_open(ctypes.byref(h), ctypes.byref(p)))
                    self._opened.append(p.value)
                    ptrs.append(p.value)
                row.append(tuple(ptrs))
            self.peers.append(row)
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.codebooks.device)

    def close(self) -> None:
        """Unmaps the peers' buffers (peer transport); collective."""
        if self.peers is None:
            return
        from . import _lib
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.check(_lib.load().ncm_ipc_close(p))
        self._opened = []
        self.peers = None

    def _barrier(self) -> None:
        dist.all_reduce(self._flag, group=self.group)

    def _push(self, b: int) -> None:
        """On the comm stream: rank r's codes [L, n] go to columns
        [r*n, (r+1)*n) of every rank's codes_out[b] (a pitched copy) and its
        reconstruction rows (encoded in place in recon_all[b]) to the same
        rows of every peer's recon_all[b]."""
        import ctypes

        from . import _lib
        lib = _lib.load()
        st = ctypes.c_void_p(self.comm.cuda_stream)
        L, n, D = self.L, self.n, self.recon_all[b].shape[1]
        es = self.recon_all[b].element_size()
        rec_off = self.rank * n * D * es
        src_rec = self.recon_all[b].data_ptr() + rec_off
        src_codes = self.codes_pad[b].data_ptr()
        self._barrier()                      # every rank's buffers of set b are free
        for k in range(1, self.world + 1):
            r = (self.rank + k) % self.world  # staggered: rank r's first copy goes to r+1
            codes_dst, recon_dst = self.peers[b][r]
            _lib.check(lib.ncm_copy2d_async(ctypes.c_void_p(codes_dst + self.rank * n * 4), self.world * n * 4,
                                            ctypes.c_void_p(src_codes), n * 4, n * 4, L, st))
            if r != self.rank:
                _lib.check(lib.ncm_copy_async(ctypes.c_void_p(recon_dst + rec_off), ctypes.c_void_p(src_rec),
                                              n * D * es, st))
        self._barrier()                      # every rank's copies into this rank's buffers have landed

    @property
    def rows(self) -> int:
        return self.stop - self.start

    def _gather(self, b: int) -> None:
        dist.all_gather_into_tensor(self.codes_all[b], self.codes_pad[b], group=self.group)
        dist.all_gather_into_tensor(self.recon_all[b], self.recon_pad[b], group=self.group)
        self.codes_out[b].view(self.L, self.world, self.n).copy_(
            self.codes_all[b].view(self.world, self.L, self.n).permute(1, 0, 2))

    def wait(self) -> None:
        """Makes the current stream wait for the last call's all-gathers (overlap mode)."""
        if self.overlap and self.calls > 0:
            torch.cuda.current_stream().wait_event(self.gathered[(self.calls - 1) & 1])

    def __call__(self, x_local: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        valid = self.rows
        if x_local.shape[0] != valid:
            raise ValueError(f"rank {self.rank} owns rows [{self.start}, {self.stop}) but got {x_local.shape[0]}")
        b = self.calls & 1 if self.overlap else 0
        cur = torch.cuda.current_stream() if self.overlap else None
        if self.overlap and self.used[b]:
            cur.wait_event(self.gathered[b])  # this buffer set's previous gathers have finished
        # the peer transport encodes the reconstruction straight into this
        # rank's rows of the gathered output
        recon_dst = (self.recon_all[b][self.rank * self.n:(self.rank + 1) * self.n] if self.peers is not None
                     else self.recon_pad[b])
        if valid == self.n:
            self.encode(x_local, self.codebooks, self.sqnorms, self.codes_pad[b], recon_dst)
        elif valid > 0:  # short last shard: encode into dense buffers, then pad
            codes = torch.empty((self.L, valid), dtype=torch.int32, device=x_local.device)
            self.encode(x_local, self.codebooks, self.sqnorms, codes, recon_dst[:valid])
            self.codes_pad[b][:, :valid] = codes
        if self.overlap:
            self.encoded[b].record(cur)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(self.encoded[b])
                if self.peers is not None:
                    self._push(b)
                else:
                    self._gather(b)
                self.gathered[b].record(self.comm)
            self.used[b] = True
        else:
            self._gather(b)
        self.calls += 1
        return self.codes_out[b][:, : self.total], self.recon_all[b][: self.total]


def sharded_encode(x_local: torch.Tensor, codebooks: torch.Tensor, total_rows: int,
                   sqnorms: torch.Tensor | None = None, group=None,
                   encode: Callable | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """One-shot form of ShardedEncoder: returns (codes [L, total_rows] int32,
    recon [total_rows, D]) on every rank."""
    enc = ShardedEncoder(codebooks, total_rows, x_local.dtype, sqnorms, group, encode)
    codes, recon = enc(x_local)
    return codes, recon


# ----------------------------------------------------- batch-sharded tokenizer

def _device_tokenizer(x, w_in, codebooks, w_out, pool_factors, **kw):
    from . import vq
    return vq.tokenizer_forward(x, w_in, codebooks, w_out, pool_factors, **kw)


class ShardedTokenizer:
    """Multiscale tokenizer forward (R6) sharded by whole batch items.

    Every pooling window of the tokenizer lies inside one batch item, so rank
    r runs the whole forward on its items [b0, b1) of the global batch with
    no exchange, and the results are all-gathered once at the end in the
    batch order of a single-GPU forward: the codes per scale [L, B*T/f_s]
    always; with gather="all" also the reconstructions [B, T, D] and the
    outputs [B, T, Din] (with the default gather="codes" those stay this
    rank's items, as data-parallel training uses them: gathering them moves
    3 * 2 * T * D bytes per item every call). Ranks hold equally many
    (padded) items so one all_gather_into_tensor per tensor suffices; the
    last ranks may hold fewer real items, or none.

    `forward(x, w_in, codebooks, w_out, pool_factors, **kw)` returns
    (codes list, recon, y) as ncmorph_b200.vq.tokenizer_forward does, which is
    the default.
    """

    def __init__(self, batch: int, seq_len: int, pool_factors: list[int], group=None,
                 forward: Callable | None = None, gather: str = "codes"):
        if gather not in ("codes", "all"):
            raise ValueError('gather is "codes" or "all"')
        self.gather = gather
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.batch, self.T = batch, seq_len
        self.pool_factors = list(pool_factors)
        if any(seq_len % f for f in self.pool_factors):
            raise ValueError("every pool factor must divide the sequence length")
        self.forward = forward or _device_tokenizer
        self.b0, self.b1, self.nb = shard_bounds(batch, self.world, self.rank)

    @property
    def items(self) -> int:
        return self.b1 - self.b0

    def _gather(self, local: torch.Tensor, per_item: int) -> torch.Tensor:
        """[nb * per_item, ...] on every rank -> [batch * per_item, ...] in batch order."""
        out = torch.empty((self.world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        parts = []
        for r in range(self.world):
            b0, b1, _ = shard_bounds(self.batch, self.world, r)
            base = r * self.nb * per_item
            parts.append(out[base:base + (b1 - b0) * per_item])
        return torch.cat(parts, 0)

    def __call__(self, x_local: torch.Tensor, w_in: torch.Tensor, codebooks: torch.Tensor, w_out: torch.Tensor,
                 **kw) -> tuple[list[torch.Tensor], torch.Tensor, torch.Tensor]:
        if x_local.shape[0] != self.items or x_local.shape[1] != self.T:
            raise ValueError(f"rank {self.rank} owns batch items [{self.b0}, {self.b1}) of length {self.T} "
                             f"but got {tuple(x_local.shape[:2])}")
        S, L, D = codebooks.shape[0], codebooks.shape[1], codebooks.shape[-1]
        if len(self.pool_factors) != S:
            raise ValueError("one pool factor per scale is required")
        Din, dev = x_local.shape[2], x_local.device
        rows = [self.T // f for f in self.pool_factors]  # pooled rows per batch item, per scale
        per_item = sum(rows)
        # every scale's codes of an item side by side, items in order: one
        # all-gather then puts the batch order in the row order
        codes_pad = torch.zeros((self.nb, per_item, L), dtype=torch.int32, device=dev)
        if self.items > 0:
            codes, recon, y = self.forward(x_local, w_in, codebooks, w_out, self.pool_factors, **kw)
            off = 0
            for s, n in enumerate(rows):
                codes_pad[: self.items, off:off + n] = codes[s].t().reshape(self.items, n, L)
                off += n
        else:
            recon = torch.empty((0, self.T, D), dtype=torch.bfloat16, device=dev)
            y = torch.empty((0, self.T, Din), dtype=torch.bfloat16, device=dev)
        gathered = self._gather(codes_pad.view(self.nb * per_item, L), per_item).view(self.batch, per_item, L)
        codes_all = []
        off = 0
        for n in rows:
            codes_all.append(gathered[:, off:off + n].reshape(self.batch * n, L).t().contiguous())
            off += n
        if self.gather == "codes":
            return codes_all, recon, y
        recon_pad = torch.zeros((self.nb, self.T, D), dtype=torch.bfloat16, device=dev)
        y_pad = torch.zeros((self.nb, self.T, Din), dtype=torch.bfloat16, device=dev)
        recon_pad[: self.items] = recon
        y_pad[: self.items] = y
        recon_all = self._gather(recon_pad.view(self.nb * self.T, D), self.T).view(self.batch, self.T, D)
        y_all = self._gather(y_pad.view(self.nb * self.T, Din), self.T).view(self.batch, self.T, Din)
        return codes_all, recon_all, y_all


# ---------------------------------------------------------------- C ABI form
# The same sharding through the library's own NCCL communicator
# (ncm_ctx_comm_init / ncm_rvq_encode_sharded), for hosts without a
# torch.distributed process group: the caller ships the 128-byte id.

def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (call on one rank, send to all)."""
    import ctypes

    from . import _lib
    buf = (ctypes.c_uint8 * 128)()
    _lib.call("ncm_comm_unique_id", buf)
    return bytes(buf)


def comm_init(device, uid: bytes, rank: int, nranks: int) -> None:
    """Binds a communicator of `nranks` ranks to this device's context (collective)."""
    import ctypes

    from . import _lib
    from .device import context
    if len(uid) != 128:
        raise ValueError("the NCCL unique id has 128 bytes")
    buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
    _lib.call("ncm_ctx_comm_init", context(device), buf, rank, nranks)


def rvq_encode_sharded(x_local: torch.Tensor, codebooks: torch.Tensor, nranks: int,
                       sqnorms: torch.Tensor | None = None, want_recon: bool = True):
    """This rank's rows x_local [n, D] bf16 -> (codes [L, nranks*n] int32,
    recon [nranks*n, D] bf16 or None) gathered from every rank."""
    from . import _lib
    from .device import context, need, ptr, stream_of
    n, D = x_local.shape
    L, K, D2 = codebooks.shape
    if D2 != D:
        raise ValueError("codebook width differs from x")
    need(x_local, torch.bfloat16, "x_local")
    need(codebooks, torch.bfloat16, "codebooks")
    dev = x_local.device
    codes = torch.empty((L, nranks * n), dtype=torch.int32, device=dev)
    recon = torch.empty((nranks * n, D), dtype=torch.bfloat16, device=dev) if want_recon else None
    _lib.call("ncm_rvq_encode_sharded", context(dev), ptr(x_local), ptr(codebooks), ptr(sqnorms), L, ptr(codes),
              ptr(recon), n, D, K, stream_of(x_local))
    return codes, recon
