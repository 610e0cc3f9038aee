"""Multi-GPU execution of the hot path: one process per GPU.

* GEMM-rooted graphs (relu(matmul(A,B)+C), ...) shard by contiguous M-row
  panels: rank r owns rows [r0, r1) of A, of every full-size epilogue
  operand and of the output, and runs the plan of its panel graph on its own
  device.  B is needed whole on every rank: it is broadcast once from the
  root over NCCL and stays resident.  Row-vector operands (bias) are small
  and replicated.  From host memory (`run_host_shared`), each rank copies
  only its slab of B over its own host link and an all-gather over NVLink
  completes B on every rank.  The output stays sharded; `gather_rows` all-gathers it
  when a single copy is needed.
* When B changes from call to call, it can cross NVLink inside the call:
  `broadcast_slabs` broadcasts it from the root in K slabs (contiguous row
  ranges of a row-major B) on a communication stream, one event per slab,
  and the plan runs in K slices (Kernel.run_torch_ksliced), slice j's
  launches waiting only for slab j -- so the GEMM over the first slabs
  overlaps the broadcast of the later ones.  The slices carry the fp32
  sums through the output in the same chunk order as one launch: the
  result is the same bit for bit.
* The same B can instead travel by copy engines (`CopyEngineRelay`): each
  rank pushes B's chunks to the next rank of a chain through CUDA IPC
  mappings and raises that rank's per-chunk flags with stream writes; the
  GEMM slices wait on the flags with stream waits.  No SM is used for the
  transfer, so the persistent GEMM keeps every SM while slabs arrive.
* Elementwise graphs shard by contiguous element ranges with no collective
  (range starts are multiples of 4 elements so every shard keeps 16-byte
  vector access).
* A rank-2 transpose shards by output row blocks (`transpose_blocks`):
  rank r writes rows [c0, c1) of the (cols x rows) output, which are
  columns [c0, c1) of the input -- a column panel it reads in place with
  the input's row stride; no collective.
Panel boundaries are multiples of 128 rows (the tensor-core tile height)
where the size allows, so no rank carries a partial tile in the middle.

The collectives go through torch.distributed (NCCL on GPUs, gloo in the
CPU tests).  The kernel work per rank is bafe_b200.compile_graph(...) of
the panel graph.
"""
from __future__ import annotations

from typing import Callable, List, Sequence, Tuple


def row_panels(M: int, world: int, align: int = 128) -> List[Tuple[int, int]]:
    """Contiguous row panels covering [0, M): as equal as possible, with
    boundaries rounded to multiples of `align` when M allows."""
    if world < 1:
        raise ValueError("world must be >= 1")
    unit = align if M >= align * world else 1
    units = (M + unit - 1) // unit
    out = []
    for r in range(world):
        a = (units * r) // world * unit
        b = (units * (r + 1)) // world * unit
        out.append((min(a, M), min(b, M)))
    return out


def element_ranges(n: int, world: int, align: int = 4) -> List[Tuple[int, int]]:
    """Contiguous element ranges covering [0, n), starts multiples of `align`."""
    return row_panels(n, world, align)


def transpose_blocks(cols: int, world: int, align: int = 64) -> List[Tuple[int, int]]:
    """Output row blocks of a transpose of a (rows x cols) matrix, one per
    rank: rank r writes output rows [c0, c1) = input columns [c0, c1);
    boundaries are multiples of `align` (the transpose kernel's tile) when
    the size allows."""
    return row_panels(cols, world, align)


def k_slices(K: int, align: int, first: int = 0, growth: float = 2.0, max_slices: int = 6) -> List[int]:
    """Bounds [0, k1, ..., K] of the K slabs a B broadcast is cut into:
    interior bounds are multiples of `align`; the first slab is small (its
    broadcast is the only one nothing overlaps), each next one `growth`
    times the previous (the GEMM over a slab outlasts the broadcast of the
    next, so the later, larger slabs stay hidden), at most `max_slices`
    slabs.  first = 0 picks K / 16."""
    if align <= 0 or K <= align:
        return [0, K]
    want = first if first > 0 else K // 16
    size = max(align, (want + align - 1) // align * align)
    bounds = [0]
    while len(bounds) < max_slices and bounds[-1] + size < K:
        bounds.append(bounds[-1] + size)
        size = max(align, int(size * growth) // align * align)
    bounds.append(K)
    # a last slab under half the one before joins it (a launch with little
    # work costs its pipeline fill and one more store and reload of the sums)
    if len(bounds) > 3 and 2 * (bounds[-1] - bounds[-2]) < bounds[-2] - bounds[-3]:
        del bounds[-2]
    return bounds


def k_slab_schedule(K: int, align: int, t_gemm_ms: float, t_bcast_ms: float, boundary_ms: float,
                    keep: float = 1.0, max_slices: int = 6) -> List[int]:
    """K slab bounds for a GEMM over a B that is broadcast in the same step.

    t_gemm_ms / t_bcast_ms: the GEMM over all of K and the broadcast of all
    of B, measured; keep: the fraction of the SMs the GEMM slices keep while
    a slab is in flight; boundary_ms: the cost of one more slice (its sums
    stored and reloaded).  Slab j+1 is R = t_gemm / (keep * t_bcast) times
    slab j, so its broadcast ends as slice j's GEMM does; with n slabs the
    step costs the first slab's broadcast (nothing overlaps it), the slower
    slices 0..n-2 and n-1 boundaries.  Returns the bounds of the n in
    [2, max_slices] with the least cost ([0, K] when slicing cannot help)."""
    if align <= 0 or K < 2 * align or t_bcast_ms <= 0:
        return [0, K]
    R = max(1.0, t_gemm_ms / (keep * t_bcast_ms))
    best, best_cost = [0, K], t_bcast_ms             # no slicing: the whole broadcast is exposed
    for n in range(2, max_slices + 1):
        w = [R ** j for j in range(n)]
        tot = sum(w)
        bounds, acc = [0], 0.0
        for j in range(n - 1):
            acc += K * w[j] / tot
            b = int(round(acc / align)) * align
            if b <= bounds[-1] or b >= K:
                break
            bounds.append(b)
        else:
            bounds.append(K)
            first, last = bounds[1] / K, (K - bounds[-2]) / K
            cost = t_bcast_ms * first + t_gemm_ms * (1.0 / keep - 1.0) * (1.0 - last) + (n - 1) * boundary_ms
            if cost < best_cost:
                best, best_cost = bounds, cost
    return best


def broadcast_slabs(B, bounds: Sequence[int], dist, src: int = 0, stream=None):
    """Broadcast the rows [bounds[j], bounds[j+1]) of B (row-major, shape
    (K, ...)) from `src`, slab by slab, in place.  On CUDA the broadcasts
    are issued on `stream` (a side stream) and a list of events is returned,
    event j recorded once slab j is in this rank's B; on the CPU (gloo) the
    calls complete in order and the list holds None."""
    import torch
    world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
    events = []
    on_gpu = B.is_cuda
    ctx = torch.cuda.stream(stream) if (on_gpu and stream is not None) else _null()
    with ctx:
        for j in range(len(bounds) - 1):
            slab = B[bounds[j]:bounds[j + 1]]
            if world > 1:
                w = dist.broadcast(slab, src=src, async_op=True)
                w.wait()                     # the issuing stream waits for the collective
            if on_gpu:
                ev = torch.cuda.Event()
                ev.record()
                events.append(ev)
            else:
                events.append(None)
    return events


RELAY_FLAG_WORDS = 1024               # uint32 flags per rank: one per chunk, the last = the ack
RELAY_ACK = RELAY_FLAG_WORDS - 1


def relay_chunks(slab_bounds: Sequence[int], row_bytes: int, split: int = 4,
                 min_bytes: int = 2 << 20, max_bytes: int = 16 << 20) -> Tuple[List[int], List[int]]:
    """Chunks of a copy-engine relay over K slabs of a row-major operand.

    Each slab [k_j, k_{j+1}) (rows) is cut into whole-row chunks of about
    slab/`split` bytes, clamped to [min_bytes, max_bytes]: small enough that
    a chunk crosses each hop of the chain quickly (the last rank's first
    slab waits for its chunks to pass every hop), large enough that the copy
    engines run at link speed.  Returns (byte bounds of the chunks, index of
    each slab's last chunk)."""
    bounds, last = [0], []
    for j in range(len(slab_bounds) - 1):
        rows = slab_bounds[j + 1] - slab_bounds[j]
        if rows <= 0:
            raise ValueError("slab bounds must increase")
        want = min(max(rows * row_bytes // split, min_bytes), max_bytes)
        per = max(1, want // row_bytes)
        n = (rows + per - 1) // per
        for i in range(1, n + 1):
            bounds.append((slab_bounds[j] + (rows * i) // n) * row_bytes)
        last.append(len(bounds) - 2)
    if len(bounds) - 1 > RELAY_ACK:
        raise ValueError(f"{len(bounds) - 1} relay chunks: at most {RELAY_ACK}")
    return bounds, last


class _DeviceArray:
    """A raw device allocation seen by torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class CopyEngineRelay:
    """B of a row-panel GEMM relayed down the chain of ranks 0 -> 1 -> ...
    -> N-1 by copy engines, inside each step (bafe_cuda_relay_step).

    Rank r's copy stream pushes chunk c of its B into rank r+1's B and
    raises rank r+1's flag c to the step number; rank r+1 forwards a chunk
    once its flag reaches the step, and its GEMM's K slice j waits (an event
    on a watch stream, recorded after a stream wait on the flag of slab j's
    last chunk) for slab j alone.  No SM is used for the transfer, so the
    persistent GEMM keeps every SM while later slabs are in flight.  A rank
    writes its predecessor's ack word once its GEMM and its forwarding of
    the step are done; the predecessor waits for it before overwriting the
    rank's B in the next step.  Steps are numbered from 1 and must be the
    same sequence on every rank.

    Construct with `over_ranks` (one process per GPU: buffers exchanged
    through CUDA IPC handles over `dist`) or `chain` (ranks emulated in one
    process, each with its own buffers, on any devices)."""

    def __init__(self, buf: int = 0, flags: int = 0, next_buf: int = 0, next_flags: int = 0, prev_flags: int = 0,
                 root: bool = False):
        self.buf, self.flags = int(buf), int(flags)
        self.next_buf, self.next_flags, self.prev_flags = int(next_buf), int(next_flags), int(prev_flags)
        self.root = bool(root)
        self._done = None
        self._owned, self._opened = [], []

    # ------------------------------------------------------------- setup --
    @staticmethod
    def _alloc(device: int, nbytes: int, handle=True):
        import ctypes
        from ._binding import check, lib
        ptr = ctypes.c_uint64(0)
        h = ctypes.create_string_buffer(64) if handle else None
        check(lib.bafe_cuda_relay_alloc(int(device), int(nbytes), ctypes.byref(ptr), h), "relay_alloc")
        return ptr.value, (h.raw if handle else None)

    @staticmethod
    def _open(device: int, handle: bytes) -> int:
        import ctypes
        from ._binding import check, lib
        ptr = ctypes.c_uint64(0)
        check(lib.bafe_cuda_relay_open(int(device), handle, ctypes.byref(ptr)), "relay_open")
        return ptr.value

    @classmethod
    def over_ranks(cls, shape, dist, device: int, typestr: str = "<f4", itemsize: int = 4):
        """Allocate this rank's B (shape, zeroed) and flag block, exchange
        IPC handles over `dist` (one all_gather_object, on every rank alike)
        and map the successor's B and flags and the predecessor's flags.
        -> (relay, B as a torch tensor on `device` or None, error message or
        None).  Errors do not raise: every rank gets a relay (holding what
        it allocated and mapped), so that all of them can agree on the
        outcome and then close() together."""
        import math
        import torch
        world, rank = dist.get_world_size(), dist.get_rank()
        r = cls(root=rank == 0)
        err, mine = None, None
        try:
            buf, hbuf = cls._alloc(device, math.prod(shape) * itemsize)
            r._owned.append(buf)
            flags, hflags = cls._alloc(device, 4 * RELAY_FLAG_WORDS)
            r._owned.append(flags)
            r.buf, r.flags, mine = buf, flags, (hbuf, hflags)
        except Exception as e:
            err = f"{type(e).__name__}: {e}"
        handles = [None] * world
        dist.all_gather_object(handles, mine)
        if err is None and any(h is None for h in handles):
            err = "relay allocation failed on another rank"
        if err is None:
            try:
                if rank + 1 < world:
                    r.next_buf = cls._open(device, handles[rank + 1][0])
                    r._opened.append(r.next_buf)
                    r.next_flags = cls._open(device, handles[rank + 1][1])
                    r._opened.append(r.next_flags)
                if rank > 0:
                    r.prev_flags = cls._open(device, handles[rank - 1][1])
                    r._opened.append(r.prev_flags)
            except Exception as e:
                err = f"{type(e).__name__}: {e}"
        t = None
        if r.buf:
            t = torch.as_tensor(_DeviceArray(r.buf, shape, typestr), device=torch.device("cuda", device))
        return r, t, err

    @classmethod
    def chain(cls, shape, devices: Sequence[int], typestr: str = "<f4", itemsize: int = 4):
        """Ranks emulated in one process: rank i's buffers on devices[i],
        its successor's and predecessor's used through plain pointers (one
        device, or devices with peer access).  -> (relays, B tensors)."""
        import math
        import torch
        nbytes = math.prod(shape) * itemsize
        bufs = [cls._alloc(d, nbytes, handle=False)[0] for d in devices]
        flags = [cls._alloc(d, 4 * RELAY_FLAG_WORDS, handle=False)[0] for d in devices]
        n = len(devices)
        relays = []
        for i in range(n):
            r = cls(bufs[i], flags[i], bufs[i + 1] if i + 1 < n else 0, flags[i + 1] if i + 1 < n else 0,
                    flags[i - 1] if i > 0 else 0, root=i == 0)
            r._owned = [bufs[i], flags[i]]
            relays.append(r)
        tensors = [torch.as_tensor(_DeviceArray(b, shape, typestr), device=torch.device("cuda", d))
                   for b, d in zip(bufs, devices)]
        return relays, tensors

    def close(self, dist=None) -> None:
        """Unmap the peers' buffers, then free this rank's.  Every rank must
        be done with the buffers (the caller synchronises its device; across
        processes it passes `dist`, and the ranks meet in a barrier before
        and after unmapping, so no buffer is freed while a peer maps it)."""
        from ._binding import lib
        multi = dist is not None and dist.is_initialized() and dist.get_world_size() > 1
        if multi:
            dist.barrier()
        for p in self._opened:
            lib.bafe_cuda_relay_close(p)
        if multi:
            dist.barrier()
        for p in self._owned:
            lib.bafe_cuda_relay_free(p)
        self._opened, self._owned = [], []

    def release(self, step: int) -> None:
        """Raise every flag of this rank (chunks and ack) far past `step` on
        a fresh stream, so that none of this rank's stream waits can stay
        pending -- the way out when a step did not complete in time (a peer
        failed).  The relayed contents are then garbage; close the relay."""
        import ctypes
        import torch
        from ._binding import lib
        if not self.flags:
            return
        s = torch.cuda.Stream()
        sp = ctypes.c_void_p(int(s.cuda_stream))
        v = (int(step) + (1 << 30)) & 0xFFFFFFFF
        for i in range(RELAY_FLAG_WORDS):
            lib.bafe_cuda_signal_write(self.flags + 4 * i, v, sp)

    # -------------------------------------------------------------- step --
    def send(self, step: int, chunk_bounds: Sequence[int], stream, start=None) -> None:
        """Enqueue this rank's part of step `step` on `stream` (its copy
        stream): the root after `start` (an event: the step's operand is
        ready); a forwarding rank after its successor's ack of the previous
        step, chunk by chunk as each arrives."""
        import ctypes
        import torch
        from ._binding import check, lib
        sp = ctypes.c_void_p(int(stream.cuda_stream))
        if start is not None:
            stream.wait_event(start)
        self._done = None
        if not self.next_buf:
            return
        check(lib.bafe_cuda_signal_wait(self.flags + 4 * RELAY_ACK, (step - 1) & 0xFFFFFFFF, sp), "signal_wait")
        n = len(chunk_bounds) - 1
        b = (ctypes.c_int64 * (n + 1))(*[int(x) for x in chunk_bounds])
        check(lib.bafe_cuda_relay_step(self.buf, self.flags, self.next_buf, self.next_flags, b, n,
                                       step & 0xFFFFFFFF, int(self.root), sp), "relay_step")
        self._done = torch.cuda.Event()
        self._done.record(stream)

    def ready(self, step: int, last_chunks: Sequence[int], stream) -> list:
        """Events for the GEMM's K slices: event j is recorded on `stream`
        (a watch stream) once slab j's last chunk has arrived; the root's
        slabs are resident (None)."""
        import ctypes
        import torch
        from ._binding import check, lib
        if self.root:
            return [None] * len(last_chunks)
        sp = ctypes.c_void_p(int(stream.cuda_stream))
        evs = []
        for c in last_chunks:
            check(lib.bafe_cuda_signal_wait(self.flags + 4 * int(c), step & 0xFFFFFFFF, sp), "signal_wait")
            e = torch.cuda.Event()
            e.record(stream)
            evs.append(e)
        return evs

    def finish(self, step: int, stream) -> None:
        """After this rank's GEMM of the step (enqueued on `stream`): wait
        for its forwarding, then acknowledge the step to the predecessor."""
        import ctypes
        from ._binding import check, lib
        if self._done is not None:
            stream.wait_event(self._done)
        if self.prev_flags:
            check(lib.bafe_cuda_signal_write(self.prev_flags + 4 * RELAY_ACK, step & 0xFFFFFFFF,
                                             ctypes.c_void_p(int(stream.cuda_stream))), "signal_write")


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def broadcast_resident(tensor, dist, src: int = 0):
    """Broadcast `tensor` from `src` in place (B of a sharded GEMM).  Raw
    16-bit half buffers (int16 / uint16 holding bf16 or f16 bits) travel as
    bytes: NCCL has no 16-bit integer type."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        import torch
        t = tensor
        if t.dtype in (torch.int16, getattr(torch, "uint16", torch.int16)) and t.is_contiguous():
            t = t.view(torch.uint8)
        dist.broadcast(t, src=src)
    return tensor


def gather_rows(panel, full_rows: int, dist, panels: Sequence[Tuple[int, int]]):
    """All-gather row panels into the full (full_rows, N) tensor on every rank.
    Panels may differ in height, so each rank pads to the largest panel."""
    import torch
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return panel
    h = max(b - a for a, b in panels)
    padded = torch.zeros((h,) + tuple(panel.shape[1:]), dtype=panel.dtype, device=panel.device)
    padded[: panel.shape[0]] = panel
    parts = [torch.empty_like(padded) for _ in panels]
    dist.all_gather(parts, padded)
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, panels)], dim=0)[:full_rows]


class SharedInput:
    """An input every rank reads whole (a row-sharded GEMM's B), assembled on
    each rank's device from host memory: rank r copies only its 1/world byte
    slab over its own host link, then one in-place all-gather over NCCL
    (NVLink) completes the buffer on every rank -- instead of every rank
    copying the whole input over PCIe.  The device buffer is kept for the
    next call of the same size."""

    def __init__(self, dist=None, device=None):
        self.dist = dist
        self.device = device
        self.buf = None                    # uint8, world x slab bytes

    def _world(self):
        d = self.dist
        if d is not None and d.is_initialized():
            return d.get_world_size(), d.get_rank()
        return 1, 0

    def copy_slab(self, host):
        """Copy this rank's byte slab of the host tensor `host` into the device
        buffer (enqueued on the current stream)."""
        import torch
        world, rank = self._world()
        flat = host.contiguous().view(-1).view(torch.uint8)
        n = flat.numel()
        slab = (n + world - 1) // world
        slab = (slab + 15) // 16 * 16                    # 16-byte aligned slabs
        dev = self.device if self.device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.buf is None or self.buf.numel() != world * slab or self.buf.device != torch.device(dev):
            self.buf = torch.empty(world * slab, dtype=torch.uint8, device=dev)
        self._host, self._n, self._slab = host, n, slab
        lo, hi = min(rank * slab, n), min((rank + 1) * slab, n)
        if hi > lo:
            self.buf[rank * slab: rank * slab + hi - lo].copy_(flat[lo:hi], non_blocking=True)

    def gather(self):
        """All-gather the slabs (after copy_slab); returns the device copy of
        the host tensor (same dtype and shape)."""
        world, rank = self._world()
        if world > 1:
            mine = self.buf[rank * self._slab:(rank + 1) * self._slab]
            self.dist.all_gather_into_tensor(self.buf, mine)
        return self.buf[:self._n].view(self._host.dtype).view(self._host.shape)

    def assemble(self, host):
        """Device copy of the host tensor `host` (same dtype and shape)."""
        self.copy_slab(host)
        return self.gather()


def run_host_shared(kernel, host_inputs: Sequence, host_out, shared: dict) -> None:
    """One host-pointer call of `kernel` (bafe_cuda_run_host_resident) where
    the inputs at the indices of `shared` (index -> SharedInput) are
    assembled on the device (slab copy, then all-gather); the other inputs
    and the output are host tensors, row-streamed as in a plain host call.
    The call starts once the slab copies are done: its own input copies run
    during the all-gather and its kernels wait for it (an event).
    Synchronous."""
    import torch
    for k, sh in shared.items():
        sh.copy_slab(host_inputs[k])
    slabs = torch.cuda.Event()
    slabs.record()
    dev_inputs = {k: sh.gather() for k, sh in shared.items()}
    ready = torch.cuda.Event()
    ready.record()
    slabs.synchronize()                                  # this rank's host link is free again
    ptrs = [(dev_inputs[k] if k in dev_inputs else t).data_ptr() for k, t in enumerate(host_inputs)]
    kernel.call_host_resident(ptrs + [host_out.data_ptr()], [k in dev_inputs for k in range(len(host_inputs))],
                              ready)


class RowPanelGemm:
    """A GEMM-rooted graph sharded over the ranks by M-row panels.

    build(rows) must return a GraphBuilder for a problem with `rows` rows of
    A / C / output (the other shapes fixed); inputs are given as full-size
    names -> tensors on the caller side and sliced here.
    """

    def __init__(self, build: Callable[[int], object], M: int, dist=None):
        import bafe_b200
        self.dist = dist
        world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
        rank = dist.get_rank() if dist is not None and dist.is_initialized() else 0
        self.panels = row_panels(M, world)
        self.r0, self.r1 = self.panels[rank]
        self.rows = self.r1 - self.r0
        self.kernel = bafe_b200.compile_graph(build(self.rows))

    def run(self, inputs: Sequence, out, stream=None) -> None:
        """inputs: this rank's operands in graph order (panels for row-sharded
        operands, the resident B whole); out: this rank's output panel."""
        self.kernel.run_torch(list(inputs), out, stream)
