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


def gather_row_shards(local: torch.Tensor, m_total: int, *, group=None) -> torch.Tensor:
    """All-gather the row blocks of a row-sharded [m_total, N] matrix.

    ``local`` holds this rank's rows (``matmul_row_shard``).  Shards may
    differ in size, so each is padded to the largest before one
    all_gather_into_tensor, and the padding is dropped afterwards.
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
        out = torch.empty((m_total, n), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = torch.zeros((mx, n), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    buf = torch.empty((ws * mx, n), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, padded, group=group)
    return torch.cat([buf[r * mx: r * mx + rows[r]] for r in range(ws)], dim=0)


def sharded_matmul(a_local: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None, *, m_total: int,
                   out_dtype: torch.dtype | None = None, replicate_output: bool = False, group=None) -> torch.Tensor:
    """This rank's rows of C = A @ B (+ bias); the full C when ``replicate_output``."""
    from .api import matmul

    c_local = matmul(a_local, b, bias, out_dtype=out_dtype)
    if not replicate_output:
        return c_local
    return gather_row_shards(c_local, m_total, group=group)


def sharded_vector_add(a_local: torch.Tensor, b_local: torch.Tensor) -> torch.Tensor:
    """This rank's element range of C = A + B (no collective)."""
    from .api import vector_add

    return vector_add(a_local, b_local)
