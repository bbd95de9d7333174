"""Row-block distributed CSR SpMV over the ranks of a process group: y = alpha*A*x + beta*y.

The reference's cusparseSpMV (libraries/sparse/src/cusparse_ops.mm:71-211) is a
single-device call.  Across GPUs the product has exactly one exchange step, the
vector x, so this module shards the matrix and exchanges only x:

- rows are split into contiguous blocks holding about the same number of stored
  entries (balanced by nnz, not by row count: power-law rows of up to 4096
  entries would otherwise load one rank far more than another); rank r keeps its
  row block (row offsets rebased to its first entry, global column indices) and
  the matching block of y;
- x is held in equal contiguous blocks of ceil(cols / world) entries; every call
  gathers the blocks into a full copy of x in this GPU's own memory, then runs the
  local product through the library's C ABI (cusparseSpMV) on the current stream.
  The gather is either one NCCL all_gather_into_tensor (``exchange="nccl"``) or
  the peer-memory pull of libmuda_peer (``exchange="peer"``, mb200_peer.h): every
  rank announces its block with a flag store into the other ranks' memory and pulls
  theirs over NVLink with 16-byte loads, one kernel and no collective per call.
  Only that pull kernel reads another GPU's memory; the product reads local x.

The local product is pluggable (``local_spmv``) only so that the partition and
exchange logic can be tested on CPU ranks with the gloo backend; the default is
the CUDA path, which raises if the library is not built.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable

import numpy as np


def nnz_balanced_bounds(row_offsets, parts: int) -> list[int]:
    """First row of each of `parts` contiguous row blocks (plus the row count at the
    end) such that every block holds about nnz / parts stored entries.

    row_offsets: the CSR offsets (rows + 1 entries, base already subtracted), any
    array-like of integers.  Blocks are cut at the row where the running entry count
    first reaches r * nnz / parts, so each block is within one row's length of the
    target; empty blocks are allowed when a single row outweighs a share."""
    ro = np.asarray(row_offsets, dtype=np.int64)
    rows = len(ro) - 1
    if parts < 1:
        raise ValueError("parts must be positive")
    nnz = int(ro[-1] - ro[0])
    bounds = [0]
    for r in range(1, parts):
        target = ro[0] + (nnz * r) // parts
        b = int(np.searchsorted(ro, target, side="left"))
        bounds.append(min(max(b, bounds[-1]), rows))
    bounds.append(rows)
    return bounds


def x_block(cols: int, world: int) -> int:
    """Entries of x each rank holds (the last block is padded)."""
    return (cols + world - 1) // world


def _peer_check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what} failed with status {status}")


class PeerExchange:
    """The x exchange over NVLink peer memory (libmuda_peer, mb200_peer.h).

    Each rank allocates an exchange buffer (flags + two x buffers of world * block
    floats), shares its CUDA IPC handle through the process group and maps every
    peer's buffer.  ``gather(x_local)`` runs one epoch on the current stream and
    returns the device address of the full x it produced (valid until the epoch
    after next reuses the buffer)."""

    def __init__(self, torch, dist, group, block: int):
        from muda_b200 import capi
        self.torch, self.dist, self.group = torch, dist, group
        self.L = capi.peer()
        self.world = dist.get_world_size(group) if dist is not None else 1
        self.rank = dist.get_rank(group) if dist is not None else 0
        self.block, self.count = block, block * self.world
        self.base = C.c_void_p()
        handle = (C.c_ubyte * capi.MB200_PEER_HANDLE_BYTES)()
        _peer_check(self.L.mb200PeerAlloc(self.count, C.byref(self.base), handle), "mb200PeerAlloc")
        self.bases = (C.c_void_p * self.world)()
        self._opened: list[C.c_void_p] = []
        self.bases[self.rank] = self.base
        if self.world > 1:
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device="cuda")
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine, group=group)
            for p in range(self.world):
                if p == self.rank:
                    continue
                h = (C.c_ubyte * capi.MB200_PEER_HANDLE_BYTES).from_buffer_copy(
                    parts[p].cpu().numpy().tobytes())
                pb = C.c_void_p()
                _peer_check(self.L.mb200PeerOpen(h, C.byref(pb)), "mb200PeerOpen")
                self.bases[p] = pb
                self._opened.append(pb)
            dist.barrier(group=group)  # every buffer is zeroed and mapped before use
        self.epoch = 0

    def gather(self, x_local) -> int:
        if x_local.numel() != self.block:
            raise ValueError(f"x block must hold {self.block} entries, got {x_local.numel()}")
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        stream = self.torch.cuda.current_stream().cuda_stream
        _peer_check(self.L.mb200PeerAllgather(self.bases, self.world, self.rank, self.count,
                                              self.block, self.epoch,
                                              C.c_void_p(x_local.data_ptr()), C.c_void_p(stream)),
                    "mb200PeerAllgather")
        return int(self.L.mb200PeerBuffer(self.base, self.count, self.epoch))

    def take_status(self) -> int:
        """Bit p set: a wait for rank p ran out since the last call (synchronises)."""
        st = C.c_uint(0)
        _peer_check(self.L.mb200PeerTakeStatus(self.base, C.byref(st)), "mb200PeerTakeStatus")
        return st.value

    def close(self) -> None:
        if not self.base:
            return
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier(group=self.group)  # nobody still reads a peer buffer
        for pb in self._opened:
            self.L.mb200PeerClose(pb)
        self._opened.clear()
        if self.world > 1:
            self.dist.barrier(group=self.group)  # every mapping of this buffer is closed
        self.L.mb200PeerFree(self.base)
        self.base = C.c_void_p()


class _CudaLocal:
    """cusparseSpMV on the local row block through the C ABI (handle and
    descriptors created once per vector buffer pair)."""

    def __init__(self, torch, offsets, col_ind, values, rows, cols, nnz, base):
        from muda_b200 import capi
        self.torch = torch
        self.L = capi.cusparse()  # raises LibraryMissing when the library is not built
        self.h = C.c_void_p()
        assert self.L.cusparseCreate(C.byref(self.h)) == 0
        self.mat = C.c_void_p()
        st = self.L.cusparseCreateCsr(C.byref(self.mat), rows, cols, nnz,
                                      C.c_void_p(offsets.data_ptr()),
                                      C.c_void_p(col_ind.data_ptr()),
                                      C.c_void_p(values.data_ptr()), 2, 2, base, 0)
        if st != 0:
            raise RuntimeError(f"cusparseCreateCsr failed with status {st}")
        self.rows, self.cols = rows, cols
        self._vecs: dict[tuple[int, int], tuple[C.c_void_p, C.c_void_p]] = {}

    def __call__(self, x_full, y_local, alpha: float, beta: float) -> None:
        self.at(x_full.data_ptr(), y_local, alpha, beta)

    def at(self, x_ptr: int, y_local, alpha: float, beta: float) -> None:
        """The product with x at device address x_ptr (cols floats)."""
        key = (x_ptr, y_local.data_ptr())
        if key not in self._vecs:
            vx, vy = C.c_void_p(), C.c_void_p()
            assert self.L.cusparseCreateDnVec(C.byref(vx), self.cols, C.c_void_p(x_ptr), 0) == 0
            assert self.L.cusparseCreateDnVec(C.byref(vy), self.rows,
                                              C.c_void_p(y_local.data_ptr()), 0) == 0
            self._vecs[key] = (vx, vy)
        vx, vy = self._vecs[key]
        stream = self.torch.cuda.current_stream().cuda_stream
        assert self.L.cusparseSetStream(self.h, C.c_void_p(stream)) == 0
        st = self.L.cusparseSpMV(self.h, 0, C.byref(C.c_float(alpha)), self.mat, vx,
                                 C.byref(C.c_float(beta)), vy, 0, 0, None)
        if st != 0:
            raise RuntimeError(f"cusparseSpMV failed with status {st}")

    def close(self) -> None:
        for vx, vy in self._vecs.values():
            self.L.cusparseDestroyDnVec(vx)
            self.L.cusparseDestroyDnVec(vy)
        self._vecs.clear()
        if self.mat:
            self.L.cusparseDestroySpMat(self.mat)
            self.mat = C.c_void_p()
        if self.h:
            self.L.cusparseDestroy(self.h)
            self.h = C.c_void_p()


def split_by_columns(torch, offsets, col_ind, values, base: int, lo: int, hi: int):
    """Splits a CSR block into the entries whose (0-based) column lies in [lo, hi) and
    the rest, both CSR with the same rows, entries kept in row order.  The first part's
    columns are rebased to lo (still in the index base), so that it indexes x[lo:hi]."""
    offs = offsets.to(torch.int64)
    rows = offs.numel() - 1
    nnz = int(offs[-1].item() - offs[0].item())
    cols0 = col_ind[:nnz].to(torch.int64) - base
    own = (cols0 >= lo) & (cols0 < hi)
    row_id = torch.repeat_interleave(torch.arange(rows, device=offs.device),
                                     (offs[1:] - offs[:-1]))
    parts = []
    for mask, shift in ((own, lo), (~own, 0)):
        counts = torch.bincount(row_id[mask], minlength=rows)
        o = torch.zeros(rows + 1, dtype=torch.int64, device=offs.device)
        o[1:] = torch.cumsum(counts, 0)
        c = (cols0[mask] - shift + base).to(torch.int32).contiguous()
        v = values[:nnz][mask].contiguous()
        # keep the arrays non-empty so that their device pointers are valid
        if c.numel() == 0:
            c = torch.full((1,), base, dtype=torch.int32, device=offs.device)
            v = torch.zeros(1, dtype=values.dtype, device=offs.device)
        parts.append(((o + base).to(torch.int32).contiguous(), c, v))
    return parts[0], parts[1]


class DistSpMV:
    """One rank's share of a row-block distributed CSR matrix.

    Build it with :meth:`from_full` (every rank passes the same full matrix and
    keeps its block) or directly from the local block.  ``spmv(alpha, x_local,
    beta, y_local)`` gathers x and computes this rank's rows of y.  With
    ``dist=None`` the object is a single rank (no process group, x is copied).
    ``exchange`` selects the gather: "nccl" (all_gather_into_tensor, or the gloo
    all_gather on CPU ranks) or "peer" (NVLink peer-memory pull, CUDA path only).

    With ``overlap=True`` (CUDA path) the block is split once into the entries whose
    column lies in this rank's own x block and the rest, each kept in row order.
    ``spmv`` then computes y = alpha * A_own * x_local + beta * y on a side stream
    while x is exchanged, and y = alpha * A_rest * x + y after it: the exchange is
    hidden behind the own-block product (half of the entries at 2 ranks, 1/N at N).
    Each row's sum is then formed in two parts, so y differs from the one-pass
    product in the last bits."""

    def __init__(self, torch, dist, group, *, offsets, col_ind, values, row_begin: int,
                 row_end: int, cols: int, base: int = 0,
                 local_spmv: Callable | None = None, device=None, exchange: str = "nccl",
                 overlap: bool = False, own_cols: tuple[int, int] | None = None):
        self.torch, self.dist, self.group = torch, dist, group
        self.world = dist.get_world_size(group) if dist is not None else 1
        self.rank = dist.get_rank(group) if dist is not None else 0
        self.row_begin, self.row_end = row_begin, row_end
        self.rows = row_end - row_begin
        self.cols = cols
        self.nnz = int(offsets[-1].item() - offsets[0].item()) if self.rows > 0 else 0
        self.xb = x_block(cols, self.world)
        dev = device if device is not None else offsets.device
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if exchange == "peer" and local_spmv is not None:
            raise ValueError("the peer exchange runs on the CUDA path only")
        self.exchange = exchange
        self._peer = PeerExchange(torch, dist, group, self.xb) if exchange == "peer" else None
        self._x_ptr = 0
        self.x_full = torch.zeros(self.xb * self.world if self._peer is None else 1,
                                  dtype=torch.float32, device=dev)
        self.overlap = overlap
        self._own = self._rest = None
        if local_spmv is None:
            self._local = _CudaLocal(torch, offsets, col_ind, values, self.rows, cols,
                                     self.nnz, base) if self.rows > 0 else None
        else:
            self._local = lambda x, y, a, b: local_spmv(offsets, col_ind, values, x, y, a, b)
        self._keep = (offsets, col_ind, values)
        if overlap and self.rows > 0:
            lo, hi = own_cols if own_cols is not None else (self.rank * self.xb,
                                                            min(cols, (self.rank + 1) * self.xb))
            self._own_lo, self._own_n = lo, max(hi - lo, 0)
            own, rest = split_by_columns(torch, offsets, col_ind, values, base, lo, hi)
            if local_spmv is None:
                self._own = _CudaLocal(torch, *own, self.rows, max(self._own_n, 1),
                                       int(own[0][-1].item()) - base, base)
                self._rest = _CudaLocal(torch, *rest, self.rows, cols,
                                        int(rest[0][-1].item()) - base, base)
                self._side = torch.cuda.Stream()
            else:
                self._own = lambda x, y, a, b: local_spmv(*own, x, y, a, b)
                self._rest = lambda x, y, a, b: local_spmv(*rest, x, y, a, b)
                self._side = None
            self._keep = self._keep + own + rest

    @classmethod
    def from_full(cls, torch, dist, group, row_offsets, col_ind, values, cols: int, *,
                  base: int = 0, local_spmv: Callable | None = None, exchange: str = "nccl",
                  overlap: bool = False):
        """Slices this rank's nnz-balanced row block out of the full CSR matrix (the
        same on every rank); the block's offsets are rebased so its first entry is
        entry 0 (plus the index base, which offsets and columns keep)."""
        world = dist.get_world_size(group) if dist is not None else 1
        rank = dist.get_rank(group) if dist is not None else 0
        ro_host = (row_offsets.cpu().numpy().astype(np.int64) - base)
        bounds = nnz_balanced_bounds(ro_host, world)
        r0, r1 = bounds[rank], bounds[rank + 1]
        e0, e1 = int(ro_host[r0]), int(ro_host[r1])
        # rebased to the block's first entry, still in the caller's index base
        offs = (row_offsets[r0:r1 + 1].to(torch.int64) - e0).to(torch.int32).contiguous()
        cols_l = col_ind[e0:e1].contiguous()
        vals_l = values[e0:e1].contiguous()
        obj = cls(torch, dist, group, offsets=offs, col_ind=cols_l, values=vals_l, row_begin=r0,
                  row_end=r1, cols=cols, base=base, local_spmv=local_spmv,
                  device=row_offsets.device, exchange=exchange, overlap=overlap)
        obj.bounds = bounds
        return obj

    def x_slice(self, x_global):
        """This rank's block of a full-length x (padded with zeros at the end)."""
        lo = self.rank * self.xb
        hi = min(lo + self.xb, self.cols)
        out = self.torch.zeros(self.xb, dtype=self.torch.float32, device=self.x_full.device)
        if hi > lo:
            out[:hi - lo] = x_global[lo:hi]
        return out

    def gather_x(self, x_local) -> None:
        """x_full <- concatenation of every rank's x block (the exchange step)."""
        if x_local.numel() != self.xb:
            raise ValueError(f"x block must hold {self.xb} entries, got {x_local.numel()}")
        if self._peer is not None:
            self._x_ptr = self._peer.gather(x_local)
            return
        if self.world == 1:
            self.x_full.copy_(x_local)
            return
        if self.dist.get_backend(self.group) == "nccl":
            self.dist.all_gather_into_tensor(self.x_full, x_local, group=self.group)
        else:
            parts = list(self.x_full.split(self.xb))
            self.dist.all_gather(parts, x_local, group=self.group)

    def local(self, alpha: float, beta: float, y_local) -> None:
        """This rank's rows of y from the gathered x (no communication)."""
        if self.rows == 0:
            return
        if y_local.numel() < self.rows:
            raise ValueError("y block is shorter than this rank's row block")
        if self._peer is not None:
            if not self._x_ptr:
                raise RuntimeError("gather_x must run before local with the peer exchange")
            self._local.at(self._x_ptr, y_local, alpha, beta)
            return
        self._local(self.x_full[:self.cols], y_local, alpha, beta)

    def spmv(self, alpha: float, x_local, beta: float, y_local) -> None:
        if self.overlap and self.rows > 0 and self._side is None:  # pluggable product
            self._own(x_local, y_local, alpha, beta)
            self.gather_x(x_local)
            self._rest(self.x_full[:self.cols], y_local, alpha, 1.0)
            return
        if self.overlap and self.rows > 0:
            torch = self.torch
            main = torch.cuda.current_stream()
            self._side.wait_stream(main)  # x_local and y are ready
            with torch.cuda.stream(self._side):
                # own-block columns index x_local (rebased), while x is exchanged
                self._own.at(x_local.data_ptr(), y_local, alpha, beta)
            self.gather_x(x_local)
            main.wait_stream(self._side)
            if self._peer is not None:
                self._rest.at(self._x_ptr, y_local, alpha, 1.0)
            else:
                self._rest(self.x_full[:self.cols], y_local, alpha, 1.0)
            return
        self.gather_x(x_local)
        self.local(alpha, beta, y_local)

    def close(self) -> None:
        if isinstance(self._local, _CudaLocal):
            self._local.close()
        self._local = None
        for part in (self._own, self._rest):
            if isinstance(part, _CudaLocal):
                part.close()
        self._own = self._rest = None
        if self._peer is not None:
            self._peer.close()
            self._peer = None
