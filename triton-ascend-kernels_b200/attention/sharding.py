"""Sequence / request sharding across ranks (one process per GPU) and the
output gather.

The reference is single-device (no torch.distributed anywhere in
attention/*.py).  Attention over independent sequences (prefill, sparse
prefill, compression) and independent requests (paged decode, sparse decode)
needs no exchange between them, so the multi-GPU form is: give each rank whole
sequences or whole requests, balance their cost with a greedy
longest-processing-time rule, run each rank's share with the single-GPU
functions, and gather the outputs once (NCCL all-gather on GPUs; any backend
works, the tests use gloo).
"""
import heapq

import torch
import torch.distributed as dist


def lpt_assign(costs, world):
    """Owner rank of each item.  Items in decreasing cost (ties: lower index
    first) go to the currently least-loaded rank (ties: lower rank)."""
    assert world >= 1
    heap = [(0.0, r) for r in range(world)]
    owner = [0] * len(costs)
    for i in sorted(range(len(costs)), key=lambda j: (-float(costs[j]), j)):
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + float(costs[i]), r))
    return owner


def _host_list(x):
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.cpu().tolist()]
    return [int(v) for v in x]


def prefill_costs(lengths, causal=True):
    """Score-matrix entries per sequence: L(L+1)/2 causal, L^2 otherwise."""
    return [L * (L + 1) // 2 if causal else L * L for L in lengths]


class VarlenShard:
    """One rank's share of a varlen (TND) batch.

    seq_ids      global indices of the sequences this rank owns (ascending)
    cu_seqlens   int32 [len(seq_ids) + 1] offsets of the local TND batch
    token_index  int64 [local tokens] global token row of each local row
    """

    def __init__(self, seq_ids, cu_seqlens, token_index):
        self.seq_ids = seq_ids
        self.cu_seqlens = cu_seqlens
        self.token_index = token_index

    def take(self, x):
        """Local rows of a global [T, ...] tensor."""
        return x.index_select(0, self.token_index.to(x.device))


def shard_varlen(cu_seqlens, world, rank, causal=True, costs=None):
    """Sequences of a varlen batch for `rank`, balanced by attention cost."""
    cu = _host_list(cu_seqlens)
    lengths = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    owner = lpt_assign(costs if costs is not None else prefill_costs(lengths, causal), world)
    seq_ids = [s for s in range(len(lengths)) if owner[s] == rank]
    local_cu, rows = [0], []
    for s in seq_ids:
        rows.append(torch.arange(cu[s], cu[s + 1], dtype=torch.int64))
        local_cu.append(local_cu[-1] + lengths[s])
    token_index = torch.cat(rows) if rows else torch.zeros(0, dtype=torch.int64)
    return VarlenShard(seq_ids, torch.tensor(local_cu, dtype=torch.int32), token_index)


def shard_requests(context_lens, world, rank):
    """Decode requests for `rank` (int64 indices, ascending), balanced by
    context length (the bytes each request streams)."""
    ctx = _host_list(context_lens)
    owner = lpt_assign([max(c, 1) for c in ctx], world)
    return torch.tensor([b for b in range(len(ctx)) if owner[b] == rank], dtype=torch.int64)


def gather_rows(local, index, total_rows, group=None, dst=None):
    """Gather variable-sized row blocks: rank r holds rows `index` of a
    [total_rows, ...] result -- an int64 tensor of global row numbers, or an
    int for a contiguous block starting at that row.  With dst=None every rank
    returns the whole result (all-gather); with dst=k only rank k does and the
    others return None (gather, for results too large to replicate).  Blocks
    are padded to the largest rank's row count for the collective; contiguous
    blocks are placed with one slice copy, others by index."""
    world = dist.get_world_size(group)
    me = dist.get_rank(group)
    dev = local.device
    contiguous = not isinstance(index, torch.Tensor)
    n = torch.tensor([local.shape[0], int(index) if contiguous else -1], dtype=torch.int64, device=dev)
    heads = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(heads, n, group=group)
    heads = [(int(h[0]), int(h[1])) for h in heads]
    counts = [c for c, _ in heads]
    mx = max(counts) if counts else 0
    if local.shape[0] == mx:
        pad = local.contiguous()
    else:
        pad = local.new_zeros((mx,) + tuple(local.shape[1:]))
        pad[: local.shape[0]] = local
    receive = dst is None or me == dst
    blocks = [torch.empty_like(pad) for _ in range(world)] if receive else None
    if dst is None:
        dist.all_gather(blocks, pad, group=group)
    else:
        dist.gather(pad, blocks, dst=dst, group=group)
    idxs = None
    if not all(r0 >= 0 for _, r0 in heads):
        # some rank sent an index tensor: exchange the row numbers too
        ipad = torch.full((mx,), -1, dtype=torch.int64, device=dev)
        if contiguous:
            ipad[: local.shape[0]] = torch.arange(int(index), int(index) + local.shape[0], device=dev)
        else:
            ipad[: local.shape[0]] = index.to(dev)
        idxs = [torch.empty_like(ipad) for _ in range(world)] if receive else None
        if dst is None:
            dist.all_gather(idxs, ipad, group=group)
        else:
            dist.gather(ipad, idxs, dst=dst, group=group)
    if not receive:
        return None
    full = local.new_zeros((total_rows,) + tuple(local.shape[1:]))
    for r, (blk, (c, r0)) in enumerate(zip(blocks, heads)):
        if not c:
            continue
        if idxs is None:
            full[r0:r0 + c] = blk[:c]
        else:
            full[idxs[r][:c]] = blk[:c]
    return full


def concat_rows(local, group=None, dst=None):
    """Every rank's [rows_r, ...] block, concatenated in rank order (blocks may
    differ in length): offsets are the prefix sums of the ranks' row counts.
    dst as in gather_rows."""
    world = dist.get_world_size(group)
    me = dist.get_rank(group)
    n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
    counts = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c) for c in counts]
    return gather_rows(local, sum(counts[:me]), sum(counts), group=group, dst=dst)


class PlannedGather:
    """All-gather of row blocks whose sizes every rank already knows from the
    sharding plan (``lpt_assign`` runs identically on every rank), in ONE
    collective with no count exchange and no host synchronisation.

    Rank r contributes ``counts[r]`` rows, padded to ``max(counts)``; the
    padded blocks are all-gathered into one tensor (``all_gather_into_tensor``)
    and, when ``row_index`` is given (``row_index[r]``: global row of each of
    rank r's rows), placed in global row order by one ``index_select`` with a
    precomputed index.  Without ``row_index`` the blocks are concatenated in
    rank order.  With ``dst=k`` the blocks go to rank k only (``gather``, for
    results too large to replicate) and the other ranks get None.  Buffers are
    allocated on first use and reused across calls."""

    def __init__(self, counts, row_index=None, group=None, dst=None):
        self.counts = [int(c) for c in counts]
        self.group = group
        self.dst = dst
        self.mx = max(self.counts) if self.counts else 0
        src = []  # position in the padded gather buffer of each global row
        if row_index is None:
            for r, c in enumerate(self.counts):
                src += [r * self.mx + i for i in range(c)]
        else:
            total = sum(self.counts)
            pos = [0] * total
            for r, rows in enumerate(row_index):
                rows = _host_list(rows)
                assert len(rows) == self.counts[r]
                for i, g in enumerate(rows):
                    pos[g] = r * self.mx + i
            src = pos
        self._src = torch.tensor(src, dtype=torch.int64)
        self._bufs = {}

    def _buffers(self, local):
        key = (local.device, local.dtype, tuple(local.shape[1:]))
        b = self._bufs.get(key)
        if b is None:
            world = len(self.counts)
            send = local.new_zeros((self.mx,) + tuple(local.shape[1:]))
            receive = self.dst is None or dist.get_rank(self.group) == self.dst
            recv = local.new_empty(((world if receive else 1) * self.mx,) + tuple(local.shape[1:]))
            b = (send, recv, self._src.to(local.device))
            self._bufs[key] = b
        return b

    def __call__(self, local):
        """The [sum(counts), ...] result (on every rank, or on rank dst only)."""
        send, recv, src = self._buffers(local)
        n = local.shape[0]
        if n == self.mx:
            send = local.contiguous()
        else:
            send[:n].copy_(local)
        if self.dst is None:
            dist.all_gather_into_tensor(recv, send, group=self.group)
        else:
            me = dist.get_rank(self.group)
            parts = list(recv.chunk(len(self.counts))) if me == self.dst else None
            dist.gather(send, parts, dst=self.dst, group=self.group)
            if me != self.dst:
                return None
        return recv.index_select(0, src)
