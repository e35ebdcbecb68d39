"""Source-row-sharded pricing scan over several GPUs (one process per GPU).

The reference is single-GPU (src/hello_ot/refinement/dual_feasibility.py:146,172).
Here rank r owns a contiguous block of source rows (x, a, f) and a replica of
the target cloud (y, b, g; y is broadcast once per solve, g per scan).  Each
rank runs the fused bidirectional scan on its block; the exchange steps are

  * certificate: all-reduce of (sum s+^2, sum c^2, count) and (max s+, max |c|);
  * column top-k: every rank owns a contiguous block of target columns; an
    all-to-all sends each rank's lists for a block (n/N x k scores + global source
    indices) to the block's owner, which merges them with the scan's order and tie
    rule, and an all-gather of the merged blocks gives every rank the merged n x k
    lists (each rank sends and receives about 2 (N-1)/N of one rank's lists, where
    an all-gather of the unmerged lists would move N-1 times them);
  * candidates: the row-side candidate pairs go to rank 0 alone (an all-to-all with
    every other destination empty), which assembles the reference's candidate order
    (source rows ascending, then target columns).

All collectives go through torch.distributed (NCCL over NVLink on the GPU box,
gloo in the CPU tests); kernel inputs are always local HBM.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from ._lib import check, lib, ptr, stream_handle


def row_partition(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced block [start, stop) of `total` rows for `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid world/rank")
    base, extra = divmod(int(total), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def merge_topk(vals: torch.Tensor, idx: torch.Tensor, k: int):
    """Merge `parts` top-k lists per row on the GPU: vals/idx (parts, rows, width)."""
    parts, rows, width = vals.shape
    out_v = torch.empty((rows, k), dtype=torch.float64, device=vals.device)
    out_i = torch.empty((rows, k), dtype=torch.int32, device=vals.device)
    L = lib()
    with torch.cuda.device(vals.device):
        rc = L.hb_merge_topk(ptr(vals.contiguous()), ptr(idx.to(torch.int32).contiguous()), parts, rows, width, k,
                             ptr(out_v), ptr(out_i), stream_handle(vals.device))
    check(rc)
    return out_v, out_i


@dataclass
class ShardedScanResult:
    rows: Optional[torch.Tensor]   # candidate pairs (rank 0 only when gathered)
    cols: Optional[torch.Tensor]
    stats: torch.Tensor            # [sum s+^2, sum c^2, max s+, max |c|, count], global
    col_vals: torch.Tensor         # merged column top-k (n x k), every rank
    col_idx: torch.Tensor
    row_vals: torch.Tensor         # this rank's rows (local block)
    row_idx: torch.Tensor


def _all_to_all(t: torch.Tensor, send: list, recv: list, group) -> torch.Tensor:
    """Rows [sum(send[:j]), sum(send[:j+1])) of t to rank j; the rows received from rank j
    land at [sum(recv[:j]), ...) of the result."""
    out = torch.empty((sum(recv), *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), recv, send, group=group)
    return out


def _all_gather(t: torch.Tensor, world: int, group) -> torch.Tensor:
    """(world, *t.shape) concatenation of every rank's t."""
    if world == 1:
        return t.unsqueeze(0)
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world, *t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.stack(parts)


class ShardedPricingScan:
    """Bidirectional ℓ2² pricing scan with source rows sharded across ranks.

    ``local_scan(x, y, a, b, qb, dbb, k)`` -> (row_vals, row_idx, col_vals, col_idx,
    stats5) and ``merge(vals, idx, k)`` default to the CUDA kernels; tests inject
    CPU versions to exercise the exchange logic under gloo.
    """

    def __init__(self, group=None, *, local_scan: Optional[Callable] = None, merge: Optional[Callable] = None,
                 dot_scale: float = 2.0, precision: str = "fp32", passes: Optional[int] = None,
                 exact: bool = True, ctas: Optional[int] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if local_scan is None:
            from .scan import l2sq_scan

            def local_scan(x, y, a, b, qb, dbb, k):
                return l2sq_scan(x, y, a, b, qb, dbb, k, dot_scale=dot_scale, precision=precision,
                                 passes=passes, exact=exact, ctas=ctas)
        self.local_scan = local_scan
        self.merge = merge or merge_topk
        self.time_phases = False  # set True to time the local scan and the exchange of each call
        self._marks = None

    def last_phase_ms(self):
        """(local scan ms, exchange and merge ms) of the last timed call (after a synchronize)."""
        if not self._marks:
            return None
        m = self._marks
        return m[0].elapsed_time(m[1]), m[1].elapsed_time(m[2])

    def scan(self, x_block, y, a_block, b, f_block, g, k: int, *, row_offset: int, theta: float = 0.0,
             gather_candidates: bool = True) -> ShardedScanResult:
        world, group = self.world, self.group
        marks = None
        if self.time_phases and x_block.is_cuda:  # CUDA events: local scan | exchange and merges
            marks = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            marks[0].record()
        rv, ri, cv, ci, stats = self.local_scan(x_block, y, a_block, b, f_block - a_block, g - b, k)
        if marks:
            marks[1].record()
        ci = torch.where(ci >= 0, ci + int(row_offset), ci)
        # certificate
        sums = stats[[0, 1, 4]].contiguous()
        maxs = stats[[2, 3]].contiguous()
        if world > 1:
            dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
            dist.all_reduce(maxs, op=dist.ReduceOp.MAX, group=group)
        total = torch.stack((sums[0], sums[1], maxs[0], maxs[1], sums[2]))
        # column lists: merged by the owner of each column block, then gathered
        if world > 1:
            n = cv.shape[0]
            blocks = [row_partition(n, world, r) for r in range(world)]
            sizes = [hi - lo for lo, hi in blocks]
            mine = sizes[self.rank]
            kk = cv.shape[1]
            pv = _all_to_all(cv, sizes, [mine] * world, group).view(world, mine, kk)
            pi = _all_to_all(ci.to(torch.int32), sizes, [mine] * world, group).view(world, mine, kk)
            mv, mi = self.merge(pv, pi, k)
            width = max(sizes)  # blocks differ by one row at most: pad to the widest
            bv = torch.full((width, k), float("-inf"), dtype=torch.float64, device=cv.device)
            bi = torch.full((width, k), -1, dtype=torch.int32, device=cv.device)
            bv[:mine] = mv
            bi[:mine] = mi.to(torch.int32)
            gv = _all_gather(bv, world, group)
            gi = _all_gather(bi, world, group)
            cv_m = torch.cat([gv[r, :sizes[r]] for r in range(world)])
            ci_m = torch.cat([gi[r, :sizes[r]] for r in range(world)])
        else:
            cv_m, ci_m = cv, ci
        rows = cols = None
        if gather_candidates:
            rmask = (rv > float(theta)) & (ri >= 0)
            local_rows = torch.nonzero(rmask, as_tuple=False)[:, 0] + int(row_offset)
            local_cols = ri[rmask].to(torch.int64)
            pairs = torch.stack((local_rows.to(torch.int64), local_cols))
            if world > 1:  # to rank 0 alone, in rank (= source row) order
                count = torch.tensor([pairs.shape[1]], dtype=torch.int64, device=pairs.device)
                counts = [int(c) for c in _all_gather(count, world, group).view(-1).tolist()]
                send = [pairs.shape[1] if r == 0 else 0 for r in range(world)]
                recv = counts if self.rank == 0 else [0] * world
                pairs = _all_to_all(pairs.t(), send, recv, group).t()
            if self.rank == 0:
                cmask = (cv_m > float(theta)) & (ci_m >= 0)
                d_local = torch.nonzero(cmask, as_tuple=False)[:, 0]
                d_match = ci_m[cmask].to(torch.int64)
                rows = torch.cat((pairs[0], d_match))
                cols = torch.cat((pairs[1], d_local.to(torch.int64)))
        if marks:
            marks[2].record()
            self._marks = marks
        return ShardedScanResult(rows=rows, cols=cols, stats=total, col_vals=cv_m, col_idx=ci_m, row_vals=rv,
                                 row_idx=ri)


class ShardedPairCosts:
    """Pair costs (the SDDMM of new or initial edges) with source rows sharded like the
    scan: each rank evaluates the edges whose source row lies in its block from its
    local rows and the replicated target cloud, then an all-gather of (edge position,
    cost) gives every rank the costs of all edges in the callers' order (exact: each
    edge is evaluated by exactly one rank).  The reference evaluates them on one GPU
    (src/hello_ot/costs/pairs.py:221-440 `_cost_pairs_lowrank_batched`).

    ``local_costs(kind, x_block, y, rows_local, cols, a_block, b, dot_scale)`` -> fp64
    costs defaults to the CUDA pair-cost kernel; tests inject a CPU version under gloo.
    """

    def __init__(self, group=None, *, local_costs: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if local_costs is None:
            from .pairs import pair_costs

            def local_costs(kind, x, y, rows, cols, a, b, dot_scale):
                return pair_costs(kind, x, y, rows, cols, a=a, b=b, dot_scale=dot_scale)
        self.local_costs = local_costs

    def costs(self, rows, cols, x_block, y, *, row_offset: int, a_block=None, b=None, kind: int = 3,
              dot_scale: float = 2.0) -> torch.Tensor:
        """fp64 cost of every (rows[e], cols[e]) (global source indices), on every rank."""
        world, group = self.world, self.group
        rows = rows.to(torch.int64).view(-1)
        cols = cols.to(torch.int64).view(-1)
        if rows.numel() != cols.numel():
            raise ValueError("rows and cols must have the same length")
        lo, hi = int(row_offset), int(row_offset) + int(x_block.shape[0])
        mine = torch.nonzero((rows >= lo) & (rows < hi), as_tuple=False).view(-1)
        vals = self.local_costs(kind, x_block, y, rows[mine] - lo, cols[mine], a_block, b, dot_scale)
        vals = vals.to(torch.float64).view(-1)
        out = torch.empty(rows.numel(), dtype=torch.float64, device=rows.device)
        if world == 1:
            if mine.numel() != rows.numel():
                raise ValueError("edge source rows outside this rank's block")
            out[mine] = vals
            return out
        count = torch.tensor([mine.numel()], dtype=torch.int64, device=rows.device)
        counts = _all_gather(count, world, group).view(-1)
        if int(counts.sum().item()) != rows.numel():
            raise ValueError("every edge's source row must lie in exactly one rank's block")
        width = max(int(counts.max().item()), 1)
        pos = torch.full((width,), -1, dtype=torch.int64, device=rows.device)
        val = torch.zeros(width, dtype=torch.float64, device=rows.device)
        pos[:mine.numel()] = mine
        val[:mine.numel()] = vals
        all_pos = _all_gather(pos, world, group)
        all_val = _all_gather(val, world, group)
        for r in range(world):
            c = int(counts[r])
            out[all_pos[r, :c]] = all_val[r, :c]
        return out
