"""The copy-engine relay's ordering protocol, checked on the CPU.

parallel.CopyEngineRelay enqueues stream waits, copies and flag writes
(bafe_cuda_signal_wait / bafe_cuda_relay_step / bafe_cuda_signal_write)
and records events; the GPU runs them in stream order.  Here the library
and torch's streams and events are replaced by a model that records every
enqueued operation and then executes the streams of all ranks in random
interleavings, honouring stream order, flag waits (>=, as
cuStreamWaitValue32 GEQ) and event waits (the record enqueued last when the
wait was enqueued).  Each rank's GEMM is modelled as slice reads of B's
chunks that begin after the slice's event and end later.  For chains of 2
to 5 ranks over several steps the model checks that:

* every interleaving finishes (no stream waits on a flag nobody raises);
* a slice reads only chunks holding the current step's B, at its start and
  at its end (no sender overwrote them with the next step's in between);
* a forwarding copy reads the current step's chunk.
"""
import random

import pytest

import bafe_b200.parallel as par


class FakeStream:
    def __init__(self, sim, sid):
        self.sim, self.cuda_stream, self.ops = sim, sid, []

    def wait_event(self, ev):
        self.ops.append(("wait_event", ev, len(ev.records)))


class FakeEvent:
    def __init__(self, sim):
        self.sim, self.records, self.done = sim, [], 0

    def record(self, stream=None):
        self.records.append(stream)
        stream.ops.append(("record", self))


class Sim:
    """Memory (flags, buffer chunks) plus the streams of every rank."""

    def __init__(self):
        self.flags = {}                 # address -> uint32
        self.chunks = {}                # (buffer address, chunk) -> step whose data it holds
        self.streams = {}

    def stream(self):
        s = FakeStream(self, len(self.streams) + 1)
        self.streams[s.cuda_stream] = s
        return s

    # the library calls the relay makes (same argument order as the C ABI)
    def bafe_cuda_signal_wait(self, addr, value, sp):
        self.streams[sp.value].ops.append(("wait_flag", int(addr), int(value)))
        return 0

    def bafe_cuda_signal_write(self, addr, value, sp):
        self.streams[sp.value].ops.append(("write_flag", int(addr), int(value)))
        return 0

    def bafe_cuda_relay_step(self, buf, flags, next_buf, next_flags, bounds, n, step, have, sp):
        ops = self.streams[sp.value].ops
        for c in range(n):
            if not have:
                ops.append(("wait_flag", int(flags) + 4 * c, int(step)))
            if next_buf:
                ops.append(("copy", int(buf), int(next_buf), c, int(step)))
                ops.append(("write_flag", int(next_flags) + 4 * c, int(step)))
        return 0

    def runnable(self, op):
        kind = op[0]
        if kind == "wait_flag":
            v = self.flags.get(op[1], 0)
            return ((v - op[2]) & 0xFFFFFFFF) < 0x80000000
        if kind == "wait_event":
            return op[2] == 0 or op[1].done >= op[2]
        return True

    def execute(self, op):
        kind = op[0]
        if kind == "write_flag":
            self.flags[op[1]] = op[2]
        elif kind == "record":
            op[1].done += 1
        elif kind == "copy":
            _, src, dst, c, step = op
            assert self.chunks.get((src, c)) == step, f"forwarded chunk {c} holds step {self.chunks.get((src, c))}"
            self.chunks[(dst, c)] = step
        elif kind == "produce":
            _, buf, n, step = op
            for c in range(n):
                self.chunks[(buf, c)] = step
        elif kind in ("read_begin", "read_end"):
            _, buf, cs, step = op
            for c in cs:
                assert self.chunks.get((buf, c)) == step, f"{kind}: chunk {c} holds step {self.chunks.get((buf, c))}, expected {step}"

    def run(self, rng):
        while True:
            live = [s for s in self.streams.values() if s.ops]
            if not live:
                return
            ready = [s for s in live if self.runnable(s.ops[0])]
            assert ready, "deadlock: " + ", ".join(f"{s.cuda_stream}:{s.ops[0][:3]}" for s in live)
            s = rng.choice(ready)
            self.execute(s.ops.pop(0))


@pytest.fixture
def sim(monkeypatch):
    import torch
    import bafe_b200._binding as binding
    sim = Sim()
    monkeypatch.setattr(binding, "lib", sim)
    monkeypatch.setattr(torch.cuda, "Event", lambda *a, **k: FakeEvent(sim))
    return sim


@pytest.mark.parametrize("ranks", [2, 3, 5])
@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_relay_steps_complete_and_read_only_their_own_step(sim, ranks, seed):
    rng = random.Random(seed * 31 + ranks)
    slabs = [0, 96, 480, 1152]
    chunk_bounds, last = par.relay_chunks(slabs, 512 * 4, min_bytes=64 << 10)
    n_chunks = len(chunk_bounds) - 1
    bufs = [0x1000000 * (r + 1) for r in range(ranks)]
    flags = [0x100000 * (r + 1) for r in range(ranks)]
    relays = [par.CopyEngineRelay(bufs[r], flags[r], bufs[r + 1] if r + 1 < ranks else 0,
                                  flags[r + 1] if r + 1 < ranks else 0, flags[r - 1] if r > 0 else 0, root=r == 0)
              for r in range(ranks)]
    comp = [sim.stream() for _ in range(ranks)]
    copy = [sim.stream() for _ in range(ranks)]
    watch = [sim.stream() for _ in range(ranks)]
    slab_chunks = [list(range(last[j - 1] + 1 if j else 0, last[j] + 1)) for j in range(len(last))]
    steps = 4
    # the host enqueues rank by rank, in a random rank order per step (hosts
    # of different processes run independently); stream execution then
    # interleaves freely
    for s in range(1, steps + 1):
        order = list(range(ranks))
        rng.shuffle(order)
        for r in order:
            start = None
            if r == 0:
                comp[0].ops.append(("produce", bufs[0], n_chunks, s))
                start = FakeEvent(sim)
                start.record(comp[0])
            relays[r].send(s, chunk_bounds, copy[r], start)
            evs = relays[r].ready(s, last, watch[r])
            for j, ev in enumerate(evs):                    # the K slices of this rank's GEMM
                if ev is not None:
                    comp[r].wait_event(ev)
                comp[r].ops.append(("read_begin", bufs[r], slab_chunks[j], s))
                comp[r].ops.append(("read_end", bufs[r], slab_chunks[j], s))
            relays[r].finish(s, comp[r])
    sim.run(rng)
    for r in range(ranks):
        assert all(sim.chunks[(bufs[r], c)] == steps for c in range(n_chunks))
        if r > 0:
            assert sim.flags[flags[r - 1] + 4 * par.RELAY_ACK] == steps


def test_a_missing_ack_is_a_deadlock_the_model_detects(sim):
    """A rank that never acknowledges a step leaves its predecessor's copy
    stream waiting for good: the model reports the deadlock (the GPU would
    wait; the bench's deadline and relay.release are the way out)."""
    rng = random.Random(7)
    slabs = [0, 96, 480, 1152]
    chunk_bounds, last = par.relay_chunks(slabs, 512 * 4, min_bytes=64 << 10)
    n_chunks = len(chunk_bounds) - 1
    bufs, flags = [0x1000000, 0x2000000], [0x100000, 0x200000]
    relays = [par.CopyEngineRelay(bufs[0], flags[0], bufs[1], flags[1], 0, root=True),
              par.CopyEngineRelay(bufs[1], flags[1], 0, 0, 0, root=False)]      # no prev_flags: never acks
    comp = [sim.stream(), sim.stream()]
    copy = [sim.stream(), sim.stream()]
    watch = [sim.stream(), sim.stream()]
    for s in (1, 2):
        for r in (0, 1):
            start = None
            if r == 0:
                comp[0].ops.append(("produce", bufs[0], n_chunks, s))
                start = FakeEvent(sim)
                start.record(comp[0])
            relays[r].send(s, chunk_bounds, copy[r], start)
            relays[r].ready(s, last, watch[r])
            relays[r].finish(s, comp[r])
    with pytest.raises(AssertionError, match="deadlock"):
        sim.run(rng)              # the root waits for an ack of step 1 that nobody writes


def test_the_model_catches_a_sender_that_skips_the_ack(monkeypatch):
    """Planted mistake: a sender that does not wait for the next rank's ack
    overwrites chunks that rank's GEMM is still reading, in some of the
    interleavings -- the read checks above must see it."""
    import torch
    import bafe_b200._binding as binding
    caught = 0
    for seed in range(12):
        sim = Sim()
        real = sim.bafe_cuda_signal_wait

        def no_ack_wait(addr, value, sp, real=real):
            if (int(addr) & 0xFFFFF) == 4 * par.RELAY_ACK:
                return 0
            return real(addr, value, sp)

        sim.bafe_cuda_signal_wait = no_ack_wait
        monkeypatch.setattr(binding, "lib", sim)
        monkeypatch.setattr(torch.cuda, "Event", lambda *a, sim=sim, **k: FakeEvent(sim))
        try:
            test_relay_steps_complete_and_read_only_their_own_step(sim, 3, seed)
        except AssertionError as e:
            assert "holds step" in str(e)
            caught += 1
    assert caught > 0
