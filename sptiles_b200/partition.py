"""Single-box partitioner: one process per GPU over torch.distributed.

* vector_add is sharded by contiguous element ranges (boundaries on 16-byte
  multiples, i.e. 4 fp32 elements);
* matmul is sharded by contiguous M-row blocks (boundaries on the 128-row
  tensor-core tile); B and the bias are replicated on every rank.

Neither op exchanges data while it computes.  The only collective is the
optional all-gather of C's row blocks for callers that want the full C on
every rank (``replicate_output``); it runs over the process group's backend
(NCCL over NVLink on the GPU box, gloo in the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .runtime import shard_range

VECTOR_ADD_ALIGN = 4  # elements: 16 bytes of fp32
MATMUL_ROW_ALIGN = 128  # rows: one tensor-core tile


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def vector_add_shard(n: int, world_size: int, rank: int) -> tuple[int, int]:
    """Element range [begin, end) of ``rank``."""
    return shard_range(n, world_size, rank, VECTOR_ADD_ALIGN)


def matmul_row_shard(m: int, world_size: int, rank: int) -> tuple[int, int]:
    """Row range [begin, end) of C (and A) owned by ``rank``."""
    return shard_range(m, world_size, rank, MATMUL_ROW_ALIGN)


def gather_row_shards(local: torch.Tensor, m_total: int, *, group=None, out: torch.Tensor | None = None
                      ) -> torch.Tensor:
    """All-gather the row blocks of a row-sharded [m_total, N] matrix.

    ``local`` holds this rank's rows (``matmul_row_shard``).  Equal shards
    gather straight into ``out`` (allocated if not given) with one
    all_gather_into_tensor; unequal shards are padded to the largest first
    and the padding is dropped afterwards.
    """
    rank = dist.get_rank(group)
    ws = dist.get_world_size(group)
    spans = [matmul_row_shard(m_total, ws, r) for r in range(ws)]
    rows = [e - b for b, e in spans]
    if local.shape[0] != rows[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard has {rows[rank]}")
    n = local.shape[1]
    mx = max(rows)
    if all(r == mx for r in rows):
        if out is None:
            out = torch.empty((m_total, n), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = torch.zeros((mx, n), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    buf = torch.empty((ws * mx, n), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, padded, group=group)
    full = torch.cat([buf[r * mx: r * mx + rows[r]] for r in range(ws)], dim=0)
    if out is not None:
        out.copy_(full)
        return out
    return full


def sharded_matmul(a_local: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None, *, m_total: int,
                   out_dtype: torch.dtype | None = None, replicate_output: bool = False, group=None) -> torch.Tensor:
    """This rank's rows of C = A @ B (+ bias); the full C when ``replicate_output``.

    With equal shards the GEMM writes straight into this rank's rows of the
    full C and the all-gather runs in place (each rank's send buffer is its
    own slice of the receive buffer), so nothing is copied on the GPU.
    """
    from .api import matmul

    if not replicate_output:
        return matmul(a_local, b, bias, out_dtype=out_dtype)
    rank, ws = dist.get_rank(group), dist.get_world_size(group)
    spans = [matmul_row_shard(m_total, ws, r) for r in range(ws)]
    if len({e - b0 for b0, e in spans}) == 1 and a_local.shape[0] == spans[rank][1] - spans[rank][0]:
        dt = out_dtype or a_local.dtype
        full = torch.empty((m_total, b.shape[1]), dtype=dt, device=a_local.device)
        r0, r1 = spans[rank]
        mine = full[r0:r1]
        matmul(a_local, b, bias, out=mine)
        dist.all_gather_into_tensor(full, mine, group=group)
        return full
    return gather_row_shards(matmul(a_local, b, bias, out_dtype=out_dtype), m_total, group=group)


def sharded_vector_add(a_local: torch.Tensor, b_local: torch.Tensor) -> torch.Tensor:
    """This rank's element range of C = A + B (no collective)."""
    from .api import vector_add

    return vector_add(a_local, b_local)


class _DeviceArray:
    """A raw device allocation presented to torch (no ownership)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr,
                                         "strides": None, "version": 3}


class ReplicatedOutput:
    """An [M, N] C held on every rank, with every rank's copy mapped into the others.

    The replicated-output mode of the partitioner with the all-gather fused
    into the GEMM: each rank allocates its copy (``st_alloc``), exports it
    (``st_ipc_handle``), the handles are exchanged over the process group, and
    each rank maps the other copies (``st_ipc_open``, NVLink peer memory on
    the B200 box).  :meth:`matmul` computes this rank's row block and the
    kernel's epilogue stores every finished chunk into all copies; one-
    element all-reduces on the current stream order the kernel after earlier
    work on every rank and later work on each rank after every rank's kernel.
    Call :meth:`close` on all ranks when done.
    """

    def __init__(self, m: int, n: int, dtype: torch.dtype, *, group=None):
        import ctypes

        from . import _native as N
        from .api import dtype_code
        from .runtime import context

        self.m, self.n, self.dtype, self.group = m, n, dtype, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world - 1 > 7:
            raise ValueError("at most 8 ranks share one replicated output")
        self.device = torch.cuda.current_device()
        self._ctx = context(self.device)
        self._N = N
        dtype_code(dtype)  # validates the type
        esize = torch.empty((), dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        N.check(N.lib().st_alloc(self._ctx, self.device, m * n * esize, ctypes.byref(ptr)), "st_alloc")
        self._ptr = ptr.value
        handle = (ctypes.c_uint8 * 64)()
        N.check(N.lib().st_ipc_handle(self._ctx, self.device, self._ptr, handle), "st_ipc_handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._peers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                continue
            p = ctypes.c_void_p()
            N.check(N.lib().st_ipc_open(self._ctx, self.device, (ctypes.c_uint8 * 64)(*h), ctypes.byref(p)),
                    f"st_ipc_open(rank {r})")
            self._peers.append(p.value)
        typestr = {4: "<f4", 2: "<f2"}[esize]
        t = torch.as_tensor(_DeviceArray(self._ptr, (m, n), typestr), device=f"cuda:{self.device}")
        self.tensor = t.view(dtype) if t.dtype != dtype else t
        self._flag = torch.zeros(1, device=f"cuda:{self.device}")
        self._peer_array = (ctypes.c_void_p * max(1, len(self._peers)))(*self._peers)
        self.rows = matmul_row_shard(m, self.world, self.rank)

    def matmul(self, a_local: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None, *,
               wait_for_readers: bool = True) -> torch.Tensor:
        """C = A @ B (+ bias) replicated on every rank; ``a_local`` holds this rank's rows.

        The kernel writes into the other ranks' copies, so by default a one-
        element all-reduce first orders it after all work already queued on
        every rank (readers of the previous result included).  Pass
        ``wait_for_readers=False`` only when nothing reads the copies between
        two calls.
        """
        import ctypes

        from .api import _exec_for, tensor_view

        r0, r1 = self.rows
        if a_local.shape[0] != r1 - r0:
            raise ValueError(f"rank {self.rank} holds {a_local.shape[0]} rows, its shard has {r1 - r0}")
        if wait_for_readers:
            dist.all_reduce(self._flag, group=self.group)
        ex = _exec_for(a_local)
        va, vb, vc = tensor_view(a_local), tensor_view(b), tensor_view(self.tensor)
        vbias = ctypes.byref(tensor_view(bias)) if bias is not None else None
        self._N.check(self._N.lib().st_matmul_allgather(self._ctx, ctypes.byref(va), ctypes.byref(vb), vbias,
                                                        ctypes.byref(vc), self._peer_array, len(self._peers), r0,
                                                        ctypes.byref(ex)), "st_matmul_allgather")
        # every rank's kernel (and so every write into this copy) precedes this
        dist.all_reduce(self._flag, group=self.group)
        return self.tensor

    def close(self) -> None:
        if self._ptr is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still writes into a copy
        for p in self._peers:
            self._N.lib().st_ipc_close(self._ctx, self.device, p)
        dist.barrier(group=self.group)  # nobody maps this copy any more
        self._N.lib().st_free(self._ctx, self.device, self._ptr)
        self._ptr = None
        self._peers = []


def sharded_matmul_host(a_local: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None, *, m_total: int,
                        out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None, group=None,
                        chunk_bytes: int = 16 << 20) -> torch.Tensor:
    """This rank's rows of C = A @ B (+ bias) with every operand in host memory.

    ``a_local`` (this rank's rows of A), ``b``, ``bias`` and ``out`` are CPU
    tensors, pinned for overlapped copies.  B is needed whole on every GPU but
    crosses the host link once per job: each rank copies 1/N of B's rows to
    its GPU and the slices are all-gathered over the process group (NCCL over
    NVLink).  Meanwhile A comes in ~16 MB row chunks on a copy stream, each
    chunk's GEMM runs once B is complete, and its rows of C go back on a
    third stream.  Returns ``out`` (allocated if not given) once it holds the
    result.
    """
    from .api import matmul

    if a_local.is_cuda or b.is_cuda or (out is not None and out.is_cuda):
        raise ValueError("sharded_matmul_host takes host tensors")
    rank, ws = dist.get_rank(group), dist.get_world_size(group)
    r0, r1 = matmul_row_shard(m_total, ws, rank)
    if a_local.shape[0] != r1 - r0:
        raise ValueError(f"rank {rank} holds {a_local.shape[0]} rows, its shard has {r1 - r0}")
    k, n = b.shape
    if a_local.shape[1] != k:
        raise ValueError(f"A has {a_local.shape[1]} columns, B has {k} rows")
    out_dtype = out_dtype or (out.dtype if out is not None else a_local.dtype)
    if out is None:
        out = torch.empty((a_local.shape[0], n), dtype=out_dtype, pin_memory=True)
    dev = torch.device("cuda", torch.cuda.current_device())
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    ks = -(-k // ws)  # B rows per rank (the last slices may be short or empty)
    b_dev = torch.empty((ks * ws, n), dtype=b.dtype, device=dev)
    rows = a_local.shape[0]
    a_dev = torch.empty((rows, k), dtype=a_local.dtype, device=dev)
    c_dev = torch.empty((rows, n), dtype=out_dtype, device=dev)
    chunk = max(256, (chunk_bytes // max(1, k * a_local.element_size())) // 256 * 256)
    with torch.cuda.stream(s_in):
        k0, k1 = min(k, rank * ks), min(k, (rank + 1) * ks)
        mine = b_dev[rank * ks:(rank + 1) * ks]
        if k1 > k0:
            mine[:k1 - k0].copy_(b[k0:k1], non_blocking=True)
        if k1 - k0 < ks:
            mine[max(0, k1 - k0):].zero_()
        bias_dev = bias.to(dev, non_blocking=True) if bias is not None else None
        b_ready = torch.cuda.Event()
        b_ready.record(s_in)
        a_ready = []
        for c0 in range(0, rows, chunk):
            a_dev[c0:c0 + chunk].copy_(a_local[c0:c0 + chunk], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
            a_ready.append(ev)
    main.wait_event(b_ready)  # this rank's slice of B and the bias are on the GPU
    dist.all_gather_into_tensor(b_dev, mine, group=group)
    b_full = b_dev[:k]
    for i, c0 in enumerate(range(0, rows, chunk)):
        main.wait_event(a_ready[i])
        matmul(a_dev[c0:c0 + chunk], b_full, bias_dev, out=c_dev[c0:c0 + chunk])
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            out[c0:c0 + chunk].copy_(c_dev[c0:c0 + chunk], non_blocking=True)
    main.wait_stream(s_out)
    main.synchronize()
    return out
