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
* Elementwise graphs shard by contiguous element ranges with no collective
  (range starts are multiples of 4 elements so every shard keeps 16-byte
  vector access).
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
