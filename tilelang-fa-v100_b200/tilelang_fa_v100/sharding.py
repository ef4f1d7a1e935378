"""Work partitioning across GPUs (one process per GPU).

The hot path has no exchange step: dense attention is independent per
(batch, head) pair and paged prefill / decode are independent per sequence, so a
multi-GPU run is a partition of those units with no collective on the data path
(NCCL only gathers results for checking).  The reference package has no multi-GPU
code; these helpers define the partition the benchmark and tests use.
"""
import heapq


def dense_pairs(batch, heads, world, rank):
    """Contiguous range [start, stop) of the flattened (batch, head) pairs owned by
    `rank`; pairs are numbered b * heads + h.  Sizes differ by at most one."""
    n = batch * heads
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def dense_batch_slice(batch, world, rank):
    """Batch rows [start, stop) of `rank` when whole batch rows are sharded (every head
    of a row stays on one GPU, so BSHD tensors shard without copies)."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def balance_sequences(lengths, world):
    """Longest-first greedy assignment of sequences to ranks by token count (LPT).
    Returns one sorted list of sequence indices per rank."""
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    owned = [[] for _ in range(world)]
    for idx in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        load, r = heapq.heappop(heap)
        owned[r].append(idx)
        heapq.heappush(heap, (load + int(lengths[idx]), r))
    return [sorted(o) for o in owned]


def contiguous_sequences(num_seqs, world, rank):
    """Sequences [start, stop) of `rank` for equal-length batches (paged prefill)."""
    return dense_batch_slice(num_seqs, world, rank)
