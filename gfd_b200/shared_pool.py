"""One pinned host pool shared by the rank processes of a node.

The reference's multi-GPU benchmark gives every GPU a pool of its own
(examples/05_multi_gpu_benchmark.cu:217-231); a serving process more often has one KV
pool in host memory that every GPU fetches from.  With one process per GPU that pool
has to live in memory the processes share: the owner rank creates an anonymous memfd
segment of the pool's size, the other ranks open the same segment through
/proc/<owner pid>/fd/<fd> (no named file, no /dev/shm size limit) and map it, and every
rank registers its mapping with its own context (gfd_pool_register: pinned, device
mapped), after which each GPU pulls its own blocks over its own link.

rate_shares() splits a job's blocks between ranks in proportion to each rank's
measured link rate, so that ranks on slower links get fewer blocks and all finish
together.  forward_plan() turns such a split into work when every rank still needs its
own blocks in its own memory: a rank whose share is below its need (a receiver) pulls the
head of its list, and ranks whose share is above their need (donors) pull the tail and
store it straight into the receiver's buffer over NVLink (gfd_gather_device with
GFD_GATHER_PEER_DST).
"""
import ctypes
import mmap
import os
from typing import List, Sequence


def rate_shares(rates: Sequence[float], total: int) -> List[int]:
    """Largest-remainder apportionment of `total` units in proportion to `rates`.

    Every rank with a positive rate gets at least one unit when total >= the number of
    such ranks; the shares always sum to `total`.  Ranks with a rate <= 0 get none
    (all-nonpositive rates: equal shares)."""
    n = len(rates)
    if n == 0:
        raise ValueError("rate_shares: no ranks")
    if total < 0:
        raise ValueError("rate_shares: negative total")
    pos = [max(float(r), 0.0) for r in rates]
    s = sum(pos)
    if s <= 0.0:
        pos = [1.0] * n
        s = float(n)
    exact = [total * r / s for r in pos]
    shares = [int(e) for e in exact]
    left = total - sum(shares)
    order = sorted(range(n), key=lambda i: (exact[i] - shares[i], pos[i]), reverse=True)
    for i in order[:left]:
        shares[i] += 1
    # a positive-rate rank left with nothing takes one unit from the largest share
    live = [i for i in range(n) if pos[i] > 0.0]
    if total >= len(live):
        for i in live:
            if shares[i] == 0:
                j = max(range(n), key=lambda k: shares[k])
                shares[j] -= 1
                shares[i] += 1
    return shares


def forward_plan(shares: Sequence[int], need: Sequence[int]):
    """Assigns the blocks each rank needs to the ranks that pull them.

    shares[r]: blocks rank r pulls in total; need[r]: blocks rank r's buffer receives.
    Returns (own, transfers): own[r] = how many of its own blocks rank r pulls (the head
    of its list, min(shares[r], need[r])); transfers = [(donor, receiver, first, count)]:
    the donor pulls the receiver's blocks [first, first + count) into the receiver's
    buffer.  Receivers are served in rank order, each by donors in rank order.  The
    shares must sum to the needs."""
    if len(shares) != len(need):
        raise ValueError("forward_plan: shares and needs differ in length")
    if sum(shares) != sum(need) or any(x < 0 for x in shares) or any(x < 0 for x in need):
        raise ValueError("forward_plan: shares must be non-negative and sum to the needs")
    own = [min(s, n) for s, n in zip(shares, need)]
    surplus = [s - o for s, o in zip(shares, own)]
    transfers = []
    d = 0
    for r, (n, o) in enumerate(zip(need, own)):
        first = o
        while first < n:
            while surplus[d] == 0:
                d += 1
            c = min(surplus[d], n - first)
            transfers.append((d, r, first, c))
            surplus[d] -= c
            first += c
    return own, transfers


class SharedSegment:
    """A memfd segment mapped into this process.

    Owner: SharedSegment.create(nbytes); the others: SharedSegment.attach(pid, fd, nbytes)
    with the owner's pid and fd (pid_fd()).  The owner must keep its segment open until
    every other rank has attached."""

    def __init__(self, fd: int, nbytes: int, owner: bool):
        self.fd = fd
        self.nbytes = nbytes
        self.owner = owner
        self.map = mmap.mmap(fd, nbytes, flags=mmap.MAP_SHARED, prot=mmap.PROT_READ | mmap.PROT_WRITE)
        self._anchor = ctypes.c_char.from_buffer(self.map)
        self.ptr = ctypes.addressof(self._anchor)

    @classmethod
    def create(cls, nbytes: int, name: str = "gfd_shared_pool") -> "SharedSegment":
        if nbytes <= 0:
            raise ValueError("SharedSegment: size must be positive")
        fd = os.memfd_create(name, 0)
        try:
            os.ftruncate(fd, nbytes)
            return cls(fd, nbytes, owner=True)
        except BaseException:
            os.close(fd)
            raise

    @classmethod
    def attach(cls, pid: int, fd: int, nbytes: int) -> "SharedSegment":
        mine = os.open(f"/proc/{int(pid)}/fd/{int(fd)}", os.O_RDWR)
        try:
            if os.fstat(mine).st_size < nbytes:
                raise ValueError("SharedSegment.attach: the segment is smaller than asked")
            return cls(mine, nbytes, owner=False)
        except BaseException:
            os.close(mine)
            raise

    def pid_fd(self):
        return os.getpid(), self.fd

    def close(self):
        if self.map is None:
            return
        self._anchor = None
        self.map.close()
        self.map = None
        os.close(self.fd)
        self.fd = -1
        self.ptr = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
