"""Splitting one problem across ranks (one process per GPU) without copies.

The three problems shard with no exchange step: the GEMV by rows M, the GEMM
and dual GEMM by columns N (B1 and B2 split identically so the SiLU gate stays
element-local).  ``shard_tuple`` returns the rank's part of a reference input
tuple as views (offset pointers and the full problem's strides), so the
drop-in ``custom_kernel`` functions run on it unchanged and write straight into
the rank's slice of C.  Shards are multiples of 128 rows / columns so that the
128-row scale blocks are never split.
"""
from __future__ import annotations


def shard_bounds(total: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """[start, end) of `rank`'s part of `total` in units of `align`, as even as possible."""
    assert total % align == 0, (total, align)
    units = total // align
    lo = (units * rank) // world
    hi = (units * (rank + 1)) // world
    return lo * align, hi * align


def shard_tuple(problem: str, data, world: int, rank: int):
    if world == 1:
        return data
    if problem == "gemv":
        a, b, sfa, sfb, sfa_p, sfb_p, c = data
        m0, m1 = shard_bounds(a.shape[0], world, rank)
        return (a[m0:m1], b, sfa[m0:m1], sfb, sfa_p[:, :, m0 // 128:m1 // 128], sfb_p, c[m0:m1])
    if problem == "gemm":
        a, b, sfa, sfb, sfa_p, sfb_p, c = data
        n0, n1 = shard_bounds(b.shape[0], world, rank)
        return (a, b[n0:n1], sfa, sfb[n0:n1], sfa_p, sfb_p[:, :, n0 // 128:n1 // 128], c[:, n0:n1])
    if problem == "dual":
        a, b1, b2, sfa, sfb1, sfb2, sfa_p, sfb1_p, sfb2_p, c = data
        n0, n1 = shard_bounds(b1.shape[0], world, rank)
        blk = slice(n0 // 128, n1 // 128)
        return (a, b1[n0:n1], b2[n0:n1], sfa, sfb1[n0:n1], sfb2[n0:n1], sfa_p,
                sfb1_p[:, :, blk], sfb2_p[:, :, blk], c[:, n0:n1])
    raise ValueError(problem)


def _dense(t):
    """A copy of `t` in the reference's storage order: operands / C
    [rows, cols, L] over contiguous (L, rows, cols); blocked scales
    (32, 4, rb, 4, kk, L) over contiguous (L, rb, kk, 32, 4, 4)."""
    if t.dim() == 3:
        return t.permute(2, 0, 1).contiguous().permute(1, 2, 0)
    if t.dim() == 6:
        return t.permute(5, 2, 4, 0, 1, 3).contiguous().permute(3, 4, 1, 5, 2, 0)
    return t.contiguous()


def dense_shard_tuple(problem: str, data, world: int, rank: int):
    """`shard_tuple` with every sliced tensor copied into its own dense
    buffer, so the rank's inputs and output are laid out exactly as the
    reference's generate_input lays out a problem of the shard's size (one
    contiguous run per tensor: a host <-> device copy is a single DMA)."""
    if world == 1:
        return data
    return tuple(_dense(t) for t in shard_tuple(problem, data, world, rank))


def output_slice(problem: str, shape, world: int, rank: int):
    """Index expression of the rank's part of C ([M, N, L])."""
    if problem == "gemv":
        m0, m1 = shard_bounds(shape[0], world, rank)
        return (slice(m0, m1), slice(None), slice(None))
    n0, n1 = shard_bounds(shape[1], world, rank)
    return (slice(None), slice(n0, n1), slice(None))
