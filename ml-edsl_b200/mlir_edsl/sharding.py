"""Row sharding of the dense layer across GPUs (one process per GPU).

Y[r] = act(X[r] @ W + b) depends only on row r, so rows split into
contiguous shards with no exchange; W and b are replicated. The partition is
the one the C runtime uses for its multi-device host calls (run_sharded in
csrc/runtime.cu): M // n rows each, the first M % n shards one row more.
"""
import os
from typing import List, Tuple


def row_shards(M: int, n: int) -> List[Tuple[int, int]]:
    """(first_row, rows) for each of n shards of M rows."""
    if n < 1:
        raise ValueError("n must be >= 1")
    base, rem = divmod(M, n)
    out, r0 = [], 0
    for i in range(n):
        rows = base + (1 if i < rem else 0)
        out.append((r0, rows))
        r0 += rows
    return out


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank float over the process group (identity without one).
    Used for timings: a multi-GPU step takes as long as its slowest rank."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_equal_rows(rows: int, group=None, device=None) -> None:
    """Raises ValueError on every rank unless every rank passes the same
    `rows`. The gathered transports place rank r's rows at r * rows of every
    rank's buffer and key their shared buffers by `rows`; unequal shards
    (row_shards of M % world != 0 rows) would otherwise leave ranks in
    mismatched collectives or store at offsets that disagree across ranks."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return
    on = device if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([int(rows), -int(rows)], dtype=torch.int64, device=on)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    hi, lo = int(t[0].item()), -int(t[1].item())
    if hi != lo:
        raise ValueError(f"gathered dense layer needs the same rows on every rank "
                         f"(got {lo}..{hi}); pad the shards to ceil(M / world) rows")


def slab_bounds(rows: int, slabs: int) -> List[Tuple[int, int]]:
    """[r0, r1) of `slabs` near-equal row slabs of `rows` rows (no empty slab)."""
    slabs = max(1, min(int(slabs), rows)) if rows > 0 else 1
    base, rem = divmod(rows, slabs)
    out, r0 = [], 0
    for i in range(slabs):
        r1 = r0 + base + (1 if i < rem else 0)
        out.append((r0, r1))
        r0 = r1
    return out


def gather_rows_pipelined(rows: int, N: int, compute_slab, *, slabs: int = 4, group=None,
                          device=None, dtype=None):
    """Assembles on every rank the full [world * rows, N] result of a
    row-sharded computation, rank r's rows at [r * rows, (r + 1) * rows).

    compute_slab(r0, r1, out) writes this rank's local rows [r0, r1) into
    `out` (a [r1 - r0, N] view of the full result) on the current stream.
    Slab s is then all-gathered on a separate stream while slab s + 1 is
    computed: with NCCL over NVLink the transfer overlaps the next slab's
    GEMM. Every rank must pass the same `rows`. Without a process group
    (or with one rank) it just computes.
    """
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank(group) if world > 1 else 0
    Y = torch.empty((world * rows, N), device=device, dtype=dtype)
    Yv = Y.view(world, rows, N)
    bounds = slab_bounds(rows, slabs)
    if world == 1:
        for r0, r1 in bounds:
            compute_slab(r0, r1, Yv[0, r0:r1])
        return Y
    on_gpu = Y.is_cuda
    nccl = dist.get_backend(group) == "nccl"
    comm = torch.cuda.Stream(device=Y.device) if on_gpu else None
    max_slab = max(r1 - r0 for r0, r1 in bounds)
    tmp = [torch.empty((world * max_slab * N,), device=device, dtype=dtype) for _ in range(2)]
    for s, (r0, r1) in enumerate(bounds):
        n = r1 - r0
        mine = Yv[rank, r0:r1]
        compute_slab(r0, r1, mine)
        ctx = None
        if on_gpu:
            ev = torch.cuda.Event()
            ev.record()
            comm.wait_event(ev)
            ctx = torch.cuda.stream(comm)
            ctx.__enter__()
        try:
            t = tmp[s % 2][: world * n * N].view(world, n, N)
            if nccl:
                dist.all_gather_into_tensor(t, mine, group=group)
            else:
                dist.all_gather(list(t.unbind(0)), mine, group=group)
            Yv[:, r0:r1].copy_(t)
        finally:
            if ctx is not None:
                ctx.__exit__(None, None, None)
    if on_gpu:
        torch.cuda.current_stream(Y.device).wait_stream(comm)
    return Y


class _DeviceArray:
    """A raw device buffer exposed through __cuda_array_interface__ (f32)."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4",
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None, "stream": None}


# Bounded wait of the peer barriers (ns): a rank that does not reach a
# gathered call within this time makes its peers' calls fail with
# B200_ERR_DEVICE_TIMEOUT instead of hanging.
PEER_TIMEOUT_NS = int(os.environ.get("B200_PEER_TIMEOUT_MS", "60000")) * 1_000_000


class _PeerRows:
    """Each rank's [world * rows, N] f32 output buffer, followed by its peer
    barrier flags (world 32-bit slots), allocated once per shape and mapped
    into every other rank (CUDA IPC) so that a rank can store its finished
    rows straight into all of them. Cached per (rows, N, device, group); held
    until the process exits. Calls order themselves against the peers with
    b200_peer_barrier on the caller's stream (barrier())."""

    _cache = {}

    @classmethod
    def get(cls, rows, N, device, group):
        key = (rows, N, device.index, id(group))
        if key not in cls._cache:
            cls._cache[key] = cls(rows, N, device, group)
        return cls._cache[key]

    def __init__(self, rows, N, device, group):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _native
        L = _native.lib()
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.world, self.rank = world, rank
        data = world * rows * N * 4
        self.flags_off = (data + 255) // 256 * 256
        nbytes = self.flags_off + 256
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        with torch.cuda.device(device):
            _native.check(L.b200_ipc_alloc(ctypes.byref(ptr), nbytes, handle))
            flags = torch.as_tensor(_DeviceArray(ptr.value + self.flags_off, (64,)), device=device)
            flags.zero_()
            torch.cuda.synchronize(device)
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs, err = [], ""
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == rank:
                    self.ptrs.append(ptr.value)
                    continue
                p = ctypes.c_void_p()
                rc = L.b200_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p))
                if rc != 0:
                    err = L.b200_last_error().decode(errors="replace")
                self.ptrs.append(p.value)
        # all ranks agree before any of them relies on the mappings, so that a
        # failure on one rank fails every rank the same way (no rank is left
        # waiting in a later collective)
        ok = torch.tensor([0 if err else 1], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            raise RuntimeError("CUDA IPC mapping of the peers' output buffers failed"
                               + (f": {err}" if err else " on another rank"))
        self.local = ptr.value
        self.Y = torch.as_tensor(_DeviceArray(ptr.value, (world * rows, N)), device=device)
        self.flag_ptrs = (ctypes.c_void_p * world)(*[p + self.flags_off for p in self.ptrs])
        self.epoch = 0
        # one copy stream per peer, so that the copy engines move the pushes
        # to different peers in parallel
        self.comm = [torch.cuda.Stream(device=device) for _ in range(world)]

    def barrier(self, stream):
        """Stream-ordered barrier of all ranks on `stream` (a torch stream)."""
        import ctypes
        from . import _native
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        _native.check(_native.lib().b200_peer_barrier(
            self.flag_ptrs, self.world, self.rank, self.epoch, PEER_TIMEOUT_NS,
            ctypes.c_void_p(stream.cuda_stream)))


class _McRows:
    """Each rank's [world * rows, N] f32 output buffer, followed by its peer
    barrier flags, in PyTorch symmetric memory whose buffers are bound to one
    NVSwitch multicast object (NVLS): a store to the multicast address lands
    in every rank's buffer. Cached per (rows, N, device, group); held until
    the process exits. Raises RuntimeError on every rank alike when the GPUs
    offer no multicast."""

    _cache = {}

    @classmethod
    def get(cls, rows, N, device, group):
        key = (rows, N, device.index, id(group))
        if key not in cls._cache:
            cls._cache[key] = cls(rows, N, device, group)
        return cls._cache[key]

    def __init__(self, rows, N, device, group):
        import ctypes
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        g = group if group is not None else dist.group.WORLD
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.world, self.rank = world, rank
        data = world * rows * N
        self.flags_off = (data * 4 + 255) // 256 * 256
        err = ""
        try:
            with torch.cuda.device(device):
                self.buf = symm_mem.empty(self.flags_off // 4 + 64, dtype=torch.float32,
                                          device=device)
                self.buf[self.flags_off // 4:].zero_()
                self.hdl = symm_mem.rendezvous(self.buf, g)
                torch.cuda.synchronize(device)
            if not self.hdl.multicast_ptr:
                err = "no NVSwitch multicast on this GPU"
        except Exception as ex:  # agreed below, so every rank fails alike
            err = f"symmetric memory: {ex}"[:300]
        ok = torch.tensor([0 if err else 1], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            raise RuntimeError("multicast output buffers unavailable"
                               + (f": {err}" if err else " on another rank"))
        self.ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        self.local = self.ptrs[rank]
        self.mc = int(self.hdl.multicast_ptr)
        self.Y = self.buf[:data].view(world * rows, N)
        self.flag_ptrs = (ctypes.c_void_p * world)(*[p + self.flags_off for p in self.ptrs])
        self.epoch = 0

    barrier = _PeerRows.barrier


def dense_rows_multicast(X_local, W, b, act: int, alpha: float, *, group=None):
    """The gathered dense layer through NVSwitch multicast: this rank's rows
    are computed once by b200_dense_f32_multicast, whose epilogue writes every
    finished value once to the multicast address of its rows, and the switch
    delivers it into every rank's output buffer. Ordered against the peers by
    peer barriers on the stream. Returns the full [world * rows, N] result,
    valid for work on this stream until the next call of this shape."""
    import ctypes
    import torch
    import torch.distributed as dist
    from . import _native
    L = _native.lib()
    rank = dist.get_rank(group)
    rows, K = X_local.shape
    N = W.shape[1]
    device = X_local.device
    buf = _McRows.get(rows, N, device, group)
    stream = torch.cuda.current_stream(device)
    buf.barrier(stream)  # every rank is done with its previous result
    off = rank * rows * N * 4
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    _native.check(L.b200_dense_f32_multicast(p(X_local), X_local.stride(0), p(W), W.stride(0),
                                             p(b), ctypes.c_void_p(buf.local + off), N,
                                             ctypes.c_void_p(buf.mc + off), rows, N, K, act,
                                             alpha, ctypes.c_void_p(stream.cuda_stream)))
    buf.barrier(stream)  # every rank's rows are in every buffer
    return buf.Y


def gather_rows_ce(rows: int, N: int, compute_slab, *, slabs: int = 4, group=None, device=None):
    """gather_rows_pipelined over the copy engines: each rank computes its rows
    slab by slab into its own region of a persistent IPC-shared output buffer
    and pushes every finished slab into the same region of each peer's buffer
    with cudaMemcpyAsync (peer DMA over NVLink, no SMs used) while the next
    slab computes. Returns the full [world * rows, N] result, valid until the
    next call with the same shape on this group. Needs one GPU per rank with
    peer access (NVLink/NVSwitch)."""
    import ctypes
    import torch
    import torch.distributed as dist
    from . import _native
    L = _native.lib()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    buf = _PeerRows.get(rows, N, device, group)
    stream = torch.cuda.current_stream(device)
    # every rank's earlier work on its stream (which may still read its
    # buffer) is done before any push into it
    buf.barrier(stream)
    Yv = buf.Y.view(world, rows, N)
    for r0, r1 in slab_bounds(rows, slabs):
        compute_slab(r0, r1, Yv[rank, r0:r1])
        ev = torch.cuda.Event()
        ev.record()
        off = (rank * rows + r0) * N * 4
        nbytes = (r1 - r0) * N * 4
        for p in range(world):
            if p != rank:
                buf.comm[p].wait_event(ev)
                _native.check(L.b200_memcpy_d2d_async(ctypes.c_void_p(buf.ptrs[p] + off),
                                                      ctypes.c_void_p(buf.local + off), nbytes,
                                                      ctypes.c_void_p(buf.comm[p].cuda_stream)))
    for p in range(world):  # this rank's pushes have landed in every peer ...
        if p != rank:
            stream.wait_stream(buf.comm[p])
    buf.barrier(stream)  # ... and every peer's pushes in this buffer
    return buf.Y


def fused_output_bases(ptrs, rank: int, rows: int, N: int):
    """Where rank `rank`'s rows go in the gathered [world * rows, N] f32
    result: (its own base, the same rows in every other rank's buffer).
    ptrs[r] is rank r's buffer as mapped on this device (ptrs[rank] its own);
    every buffer holds world * rows rows of N floats, this rank's at row
    rank * rows."""
    off = rank * rows * N * 4
    return ptrs[rank] + off, [p + off for r, p in enumerate(ptrs) if r != rank]


def dense_rows_fused(X_local, W, b, act: int, alpha: float, *, group=None):
    """The gathered dense layer with the collective inside the GEMM: this
    rank's rows are computed once by b200_dense_f32_peers, whose epilogue
    stores every finished value both into this rank's region of its own
    persistent IPC-shared output buffer and into the same region of every
    peer's buffer (stores over NVLink while later tiles compute; no copy
    pass). Returns the full [world * rows, N] result, valid until the next
    call with the same shape on this group."""
    import ctypes
    import torch
    import torch.distributed as dist
    from . import _native
    L = _native.lib()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rows, K = X_local.shape
    N = W.shape[1]
    if world - 1 > 7:
        raise ValueError("the fused transport stores into at most 7 peers")
    device = X_local.device
    buf = _PeerRows.get(rows, N, device, group)
    stream = torch.cuda.current_stream(device)
    # every rank's earlier work on its stream (which may still read its
    # buffer) is done before any store into it
    buf.barrier(stream)
    own, peers = fused_output_bases(buf.ptrs, rank, rows, N)
    arr = (ctypes.c_void_p * max(1, len(peers)))(*peers)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    st = ctypes.c_void_p(stream.cuda_stream)
    _native.check(L.b200_dense_f32_peers(p(X_local), X_local.stride(0), p(W), W.stride(0), p(b),
                                         ctypes.c_void_p(own), N, arr, len(peers),
                                         rows, N, K, act, alpha, st))
    # this rank's stores have landed in every peer, and every peer's in this
    # buffer, before later work on the stream reads it
    buf.barrier(stream)
    return buf.Y


def dense_rows(X_local, W, b=None, act: int = 1, alpha: float = 0.0, *, gather: bool = False,
               slabs: int = 4, group=None, reserve_sms: int = 8, transport: str = "ce"):
    """Y = act(X_local @ W + b) for this rank's rows on its GPU (torch f32
    CUDA tensors, rows of X_local contiguous), through the B200 C-ABI on the
    current stream. gather=False returns this rank's rows (no communication);
    gather=True returns the full result on every rank, all-gathered with NCCL
    over NVLink slab by slab while later slabs compute (every rank must hold
    the same number of rows). transport "multimem" has the GEMM's epilogue
    write every finished value once to an NVSwitch multicast address that
    reaches all ranks' buffers (see dense_rows_multicast); "ce" pushes finished slabs into the
    peers' IPC-mapped output buffers with the copy engines (no SMs, overlaps
    the next slab's GEMM; the result is a persistent buffer valid until the
    next call of this shape); "fused" has the GEMM's epilogue store every
    finished tile into the peers' buffers directly (one launch sequence, no
    slabs; see dense_rows_fused); "nccl" all-gathers each slab with NCCL on a
    side stream, with the GEMM's grid leaving `reserve_sms` SMs free for
    NCCL's kernels (cap NCCL's CTAs to match, e.g. NCCL_MAX_CTAS)."""
    import ctypes
    import torch
    from . import _native
    L = _native.lib()
    M, K = X_local.shape
    N = W.shape[1]
    if X_local.stride(1) != 1 or W.stride(1) != 1:
        raise ValueError("X_local and W need contiguous rows")
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None

    def compute(r0, r1, out):
        st = ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)
        Xs = X_local[r0:r1]
        _native.check(L.b200_dense_f32(p(Xs), Xs.stride(0), p(W), W.stride(0), p(b), p(out),
                                       out.stride(0), r1 - r0, N, K, act, alpha, st))

    if not gather:
        Y = torch.empty((M, N), device=X_local.device, dtype=torch.float32)
        compute(0, M, Y)
        return Y
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    if transport not in ("ce", "nccl", "fused", "multimem"):
        raise ValueError(f"unknown transport {transport!r}")
    check_equal_rows(M, group, X_local.device)
    if transport == "multimem" and world > 1:
        if K == 0:
            raise ValueError("the multimem transport needs K > 0")
        return dense_rows_multicast(X_local, W, b, act, alpha, group=group)
    if transport == "fused" and world > 1:
        return dense_rows_fused(X_local, W, b, act, alpha, group=group)
    if transport == "ce" and world > 1:
        return gather_rows_ce(M, N, compute, slabs=slabs, group=group, device=X_local.device)
    limit = 0
    if world > 1 and reserve_sms > 0:
        sms = torch.cuda.get_device_properties(X_local.device).multi_processor_count
        limit = max(1, sms - int(reserve_sms))
    prev = L.b200_set_gemm_sm_limit(limit)
    try:
        return gather_rows_pipelined(M, N, compute, slabs=slabs, group=group,
                                     device=X_local.device, dtype=torch.float32)
    finally:
        L.b200_set_gemm_sm_limit(max(prev, 0))
