"""CPU model of the GEMM kernel's barrier protocol, run under randomised schedules (test infrastructure).

It restates, role by role, what ``cutex_b200/csrc/mxfp8_gemm.cuh`` does with
its mbarriers, and checks the data hazards the protocol exists to prevent:

* the shared-memory ring (``full``/``empty`` per stage): the producer waits
  ``empty[s]`` with parity ``((kit / S) & 1) ^ 1``, the leader posts the
  expected bytes of the whole (pair) stage and every CTA's copies complete on
  the leader's ``full[s]``; the MMA issuer waits ``full[s]`` with parity
  ``(kit / S) & 1``, queues the scale copies and four MMAs on the tensor pipe and
  commits ``empty[s]`` of every CTA (kernel: producer and MMA loops);
* the TMEM accumulators (``acc_full``/``acc_empty`` per buffer, count
  ``4 * cta_group``): two buffers alternate by tile; when two tiles plus the
  scale columns exceed 512 columns, buffer 1 overlaps the end of buffer 0 and
  the MMA issuer of tile ``it`` waits for tile ``it - 1``'s release, which the
  epilogue warps post after reading the overlapping chunk first (``GemmCfg``:
  ``kOverlap``, ``kAcc1Col``, ``kFirstChunk0``);
* the rotating scale-factor TMEM buffers (``kit % sf_bufs``).

Asynchronous agents are modelled explicitly: a TMA copy lands at a random later
time; the tensor pipe executes its queue in issue order, one operation at a
time, and a commit arrives once everything queued before it has executed.
Each shared-memory stage and each TMEM column records who wrote it last and
who still has to read it; a write over unread data, a read of stale data, or a
state where nothing can advance before every role has finished (deadlock) is
a protocol error. ``Mutation`` plants known mistakes so the tests can show the
checker catches them.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field

TMEM_COLS = 512
SF_BUF_COLS = 16


class ProtocolError(AssertionError):
    pass


@dataclass(frozen=True)
class Shape:
    """One kernel instantiation and problem: (cta_group, tile_n, stages, sf_bufs), tiles per CTA, K-stages."""

    cta_group: int
    tile_n: int
    stages: int
    sf_bufs: int
    tiles: int
    k_blocks: int

    @property
    def sf_reserved(self) -> int:
        return SF_BUF_COLS * self.sf_bufs

    @property
    def overlap(self) -> bool:
        return 2 * self.tile_n + self.sf_reserved > TMEM_COLS

    @property
    def acc1_col(self) -> int:
        return TMEM_COLS - self.sf_reserved - self.tile_n if self.overlap else self.tile_n

    @property
    def sf_col(self) -> int:
        return TMEM_COLS - self.sf_reserved if self.overlap else 2 * self.tile_n

    @property
    def chunks(self) -> int:
        return self.tile_n // 64

    def acc_cols(self, buf: int) -> range:
        start = self.acc1_col if buf else 0
        return range(start, start + self.tile_n)

    def first_chunk(self, buf: int) -> int:
        return self.acc1_col // 64 if (self.overlap and buf == 0) else 0


@dataclass
class Mutation:
    """Deliberate protocol mistakes (all off by default)."""

    mma_waits_own_buffer: bool = False      # overlap build: wait for tile it-2's release instead of it-1's
    release_after_first_chunk_only: bool = False  # non-overlap build: release before reading the tile
    epilogue_skips_overlap_first: bool = False  # overlap build: read chunks in order 0..n-1, release after chunk 0
    producer_parity_unflipped: bool = False  # producer waits empty with parity (kit/S)&1
    commit_before_last_mma: bool = False     # empty[s] committed before the stage's last MMA is queued


class Barrier:
    """An mbarrier: arrival count, transaction bytes, phase; try_wait(parity) as in PTX."""

    def __init__(self, count: int, name: str):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0
        self.name = name

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, expect_tx: int = 0):
        if self.pending <= 0:
            raise ProtocolError(f"{self.name}: arrival beyond the expected count")
        self.tx += expect_tx
        self.pending -= 1
        self._maybe_complete()

    def complete_tx(self, nbytes: int):
        # A copy may land before the expected bytes are posted (the count goes
        # negative); the phase cannot complete then, an arrival is still pending.
        self.tx -= nbytes
        self._maybe_complete()

    def passed(self, parity: int) -> bool:
        return (self.phase & 1) != parity


@dataclass
class Stage:
    kit: int = -1          # K-stage whose data the stage holds (after its copy landed)
    writing: int = -1      # K-stage whose copy is in flight
    readers: int = 0       # pipe operations queued on this stage and not yet executed


@dataclass
class Column:
    tile: int = -1         # tile whose accumulation the column holds
    unread: int = 0        # epilogue warps that still have to read it for that tile
    sf_kit: int = -1       # scale-factor columns: K-stage whose scales they hold
    sf_unread: int = 0     # MMAs that still have to read them


@dataclass
class Sim:
    shape: Shape
    rng: random.Random
    mut: Mutation = field(default_factory=Mutation)

    def __post_init__(self):
        sh = self.shape
        cg = sh.cta_group
        self.full = [Barrier(1, f"full[{s}]") for s in range(sh.stages)]  # leader's
        self.empty = [[Barrier(1, f"cta{r}.empty[{s}]") for s in range(sh.stages)] for r in range(cg)]
        self.acc_full = [[Barrier(1, f"cta{r}.acc_full[{b}]") for b in range(2)] for r in range(cg)]
        self.acc_empty = [Barrier(4 * cg, f"acc_empty[{b}]") for b in range(2)]  # leader's
        self.smem = [[Stage() for _ in range(sh.stages)] for _ in range(cg)]
        self.tmem = [[Column() for _ in range(TMEM_COLS)] for _ in range(cg)]
        self.stage_bytes = 1000  # any per-CTA byte count: expect-tx is stage_bytes * cta_group
        self.pipe: list[tuple] = []    # tensor pipe queue (in issue order)
        self.landing: list[tuple] = []  # TMA copies in flight: (cta, stage, kit)
        self.tiles_done = [0] * cg      # tiles every epilogue warp of a CTA has finished
        self.mma_tile_ops: dict[int, int] = {}  # tile -> MMA operations not yet executed
        self.roles = []
        for r in range(cg):
            self.roles.append(self._producer(r))
        self.roles.append(self._mma())
        for r in range(cg):
            for w in range(4):
                self.roles.append(self._epilogue(r, w))

    # ---------------------------------------------------------------- roles (generators yield a wait predicate)

    def _producer(self, r):
        sh = self.shape
        kit = 0
        for _t in range(sh.tiles):
            for _kb in range(sh.k_blocks):
                s = kit % sh.stages
                parity = ((kit // sh.stages) & 1) ^ (0 if self.mut.producer_parity_unflipped else 1)
                yield lambda s=s, p=parity: self.empty[r][s].passed(p)
                st = self.smem[r][s]
                if st.readers:
                    raise ProtocolError(f"cta{r} stage {s}: copy of K-stage {kit} issued over data the pipe "
                                        f"still has to read (K-stage {st.kit})")
                if r == 0:
                    self.full[s].arrive(expect_tx=self.stage_bytes * sh.cta_group)
                st.writing = kit
                self.landing.append((r, s, kit))
                kit += 1
        for i in range(sh.stages):  # drain: every filled stage consumed before exit
            k2 = kit + i
            yield lambda s=k2 % sh.stages, p=((k2 // sh.stages) & 1) ^ 1: self.empty[r][s].passed(p)

    def _mma(self):
        sh = self.shape
        kit = 0
        for it in range(sh.tiles):
            buf = it & 1
            if sh.overlap and not self.mut.mma_waits_own_buffer:
                if it >= 1:
                    prev = it - 1
                    yield lambda b=prev & 1, p=(prev >> 1) & 1: self.acc_empty[b].passed(p)
            else:
                if it >= 2:
                    yield lambda b=buf, p=((it - 2) >> 1) & 1: self.acc_empty[b].passed(p)
            self.mma_tile_ops[it] = 0
            for _kb in range(sh.k_blocks):
                s = kit % sh.stages
                yield lambda s=s, p=(kit // sh.stages) & 1: self.full[s].passed(p)
                for r in range(sh.cta_group):
                    if self.smem[r][s].kit != kit:
                        raise ProtocolError(f"MMA of K-stage {kit} found cta{r} stage {s} holding "
                                            f"K-stage {self.smem[r][s].kit}")
                sf = sh.sf_col + (kit % sh.sf_bufs) * SF_BUF_COLS
                self.pipe.append(("sf_copy", kit, s, sf))
                for r in range(sh.cta_group):
                    self.smem[r][s].readers += 5
                ops = [("mma", kit, s, sf, it, buf) for _ in range(4)]
                if self.mut.commit_before_last_mma:
                    self.pipe.extend(ops[:3])
                    self.pipe.append(("commit_empty", s))
                    self.pipe.append(ops[3])
                else:
                    self.pipe.extend(ops)
                    self.pipe.append(("commit_empty", s))
                self.mma_tile_ops[it] += 4
                kit += 1
            self.pipe.append(("commit_acc", it, buf))

    def _epilogue(self, r, w):
        sh = self.shape
        for it in range(sh.tiles):
            buf = it & 1
            yield lambda b=buf, p=(it >> 1) & 1: self.acc_full[r][b].passed(p)
            if self.mma_tile_ops.get(it, 1) != 0:
                raise ProtocolError(f"cta{r} warp {w}: tile {it}'s accumulator signalled before its MMAs ran")
            first = 0 if self.mut.epilogue_skips_overlap_first else sh.first_chunk(buf)
            base = sh.acc_cols(buf).start
            for i in range(sh.chunks):
                c = (first + i) % sh.chunks
                yield lambda: True  # the chunk's TMEM load takes its time
                for col in range(base + 64 * c, base + 64 * c + 64):
                    cell = self.tmem[r][col]
                    if cell.tile != it:
                        raise ProtocolError(f"cta{r} warp {w}: column {col} holds tile {cell.tile}, "
                                            f"expected tile {it}")
                    cell.unread -= 1
                if sh.overlap or self.mut.epilogue_skips_overlap_first:
                    release = i == 0
                else:
                    release = i == 0 if self.mut.release_after_first_chunk_only else i == sh.chunks - 1
                if release:
                    self.acc_empty[buf].arrive()

    # ---------------------------------------------------------------- asynchronous agents

    def _land_copy(self):
        r, s, kit = self.landing.pop(self.rng.randrange(len(self.landing)))
        if self.full[s].phase != kit // self.shape.stages:
            raise ProtocolError(f"cta{r}: bytes of K-stage {kit} landed on phase {self.full[s].phase} of full[{s}]")
        st = self.smem[r][s]
        st.kit, st.writing = kit, -1
        self.full[s].complete_tx(self.stage_bytes)

    def _pipe_step(self):
        op = self.pipe.pop(0)
        sh = self.shape
        kind = op[0]
        if kind == "sf_copy":
            _, kit, s, sf = op
            for r in range(sh.cta_group):
                for col in range(sf, sf + SF_BUF_COLS):
                    cell = self.tmem[r][col]
                    if cell.sf_unread:
                        raise ProtocolError(f"scale columns {sf}+ overwritten before K-stage {cell.sf_kit}'s MMAs")
                    cell.sf_kit, cell.sf_unread = kit, 4
                self.smem[r][s].readers -= 1
        elif kind == "mma":
            _, kit, s, sf, it, buf = op
            for r in range(sh.cta_group):
                if self.smem[r][s].kit != kit:
                    raise ProtocolError(f"MMA of K-stage {kit} read cta{r} stage {s} after it was overwritten")
                self.smem[r][s].readers -= 1
                if self.tmem[r][sf].sf_kit != kit:
                    raise ProtocolError(f"MMA of K-stage {kit} read scales of K-stage {self.tmem[r][sf].sf_kit}")
                for col in range(sf, sf + SF_BUF_COLS):
                    self.tmem[r][col].sf_unread -= 1
                for col in sh.acc_cols(buf):
                    cell = self.tmem[r][col]
                    if cell.tile != it:
                        if cell.unread:
                            raise ProtocolError(f"cta{r}: tile {it}'s MMA overwrote column {col} before the "
                                                f"epilogue read tile {cell.tile}")
                        cell.tile, cell.unread = it, 4
            self.mma_tile_ops[it] -= 1
        elif kind == "commit_empty":
            for r in range(sh.cta_group):
                self.empty[r][op[1]].arrive()
        elif kind == "commit_acc":
            for r in range(sh.cta_group):
                self.acc_full[r][op[2]].arrive()

    # ---------------------------------------------------------------- scheduler

    def run(self, max_steps: int = 200000) -> None:
        waiting = [None] * len(self.roles)  # predicate each role waits on (None: runnable)
        done = [False] * len(self.roles)
        # Each agent gets its own speed for the whole run (a slow epilogue warp, a
        # fast tensor pipe, ...), so skewed interleavings are explored, not only
        # ones where every agent advances at the same average rate.
        speed = {("role", i): self.rng.choice((0.02, 0.2, 1.0)) for i in range(len(self.roles))}
        speed[("land", None)] = self.rng.choice((0.02, 0.2, 1.0))
        speed[("pipe", None)] = self.rng.choice((0.02, 0.2, 1.0))
        for _ in range(max_steps):
            runnable = [i for i, role in enumerate(self.roles)
                        if not done[i] and (waiting[i] is None or waiting[i]())]
            choices = [("role", i) for i in runnable]
            if self.landing:
                choices.append(("land", None))
            if self.pipe:
                choices.append(("pipe", None))
            if not choices:
                if all(done):
                    return
                stuck = [i for i in range(len(self.roles)) if not done[i]]
                raise ProtocolError(f"deadlock: roles {stuck} wait and nothing is in flight")
            kind, i = self.rng.choices(choices, weights=[speed[c] for c in choices])[0]
            if kind == "land":
                self._land_copy()
            elif kind == "pipe":
                self._pipe_step()
            else:
                try:
                    waiting[i] = next(self.roles[i])
                except StopIteration:
                    done[i] = True
                    waiting[i] = None
        raise ProtocolError("the simulation did not finish")


def simulate(shape: Shape, seed: int, mutation: Mutation | None = None) -> None:
    Sim(shape, random.Random(seed), mutation or Mutation()).run()
