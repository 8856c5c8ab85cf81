"""Disaggregated serving on one node: prefill GPU groups stream every request's KV cache, one
request at a time, into a decode GPU group's continuous batcher over NVLink.

Topology (`Split`): ranks [0, P) form P / tp prefill groups and ranks [P, N) form (N - P) / tp
decode groups, each group a tensor-parallel set of tp consecutive ranks (Megatron layout, NCCL
all-reduce inside the group). Decode group j is fed by prefill group j mod (P / tp), and TP
rank t of a prefill group hands its KV-head shard to TP rank t of each decode group it feeds
(the reference's equal-TP pairing, hexgen/llama/llama_disaggregate_with_tp_test.py:161, :170;
each rank's cache already holds only its own heads, mha.py:598-599).

Per request (the reference hands off per request too, hexgen2/run.py:141-198):
  prefill rank   prefill at batch 1 (Engine.prefill's flow) -> greedy first token (with TP one
                 all-reduce of (value, index) keys) -> one gather-pack launch writes the live
                 rows of every layer straight into the decode rank's staging ring (peer stores
                 over NVLink into a CUDA-IPC mapping) -> stream sync -> publishes
                 {first token, length, ring offset} under a store key;
  decode rank    between decode steps, admits ready requests into free slots of its
                 ContinuousBatcher (one scatter launch each, from its own local ring), decodes
                 every slot with one replay of the kept decode graph, retires finished requests,
                 and publishes which ring regions it has consumed.
The staging ring is a byte ring written in request order; the prefill rank waits for the decode
rank's "consumed" key of the oldest overlapping region before reusing its bytes, so a pack never
overwrites rows that have not been scattered yet. Control messages are small keys in the process
group's TCP store; only KV bytes travel over NVLink. Within a TP decode group the leader (TP
rank 0) decides each step's admissions and publishes them, so every rank admits the same
requests into the same slots and the TP collectives inside the decode graph stay in step.

Requests are admitted in their decode group's order as soon as all TP shards are staged, so
prefill of later requests overlaps decoding of earlier ones; a decode group never waits for a
whole batch.
"""
from __future__ import annotations

import json
import time
from collections import deque
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops
from .engine import PREFILL_PROMPTS, PREFILL_TOKENS, ContinuousBatcher
from .transport import KVHandoff

ALIGN = 256  # ring offsets: 16 B suffices for the copy kernels; 256 keeps regions apart


@dataclass
class Split:
    """world ranks -> prefill groups [0, prefill_gpus) and decode groups [prefill_gpus, world),
    tensor-parallel groups of `tp` consecutive ranks."""
    world: int
    prefill_gpus: int
    tp: int = 1

    def __post_init__(self):
        d = self.world - self.prefill_gpus
        if (self.tp < 1 or self.prefill_gpus < self.tp or d < self.tp
                or self.prefill_gpus % self.tp or d % self.tp):
            raise ValueError(f"cannot split {self.world} GPUs into {self.prefill_gpus} prefill + "
                             f"{d} decode GPUs in tensor-parallel groups of {self.tp}")

    @classmethod
    def for_throughput(cls, world: int, tp: int = 1) -> "Split":
        """About one prefill GPU per three decode GPUs (a Llama-2-7B decode of 32 requests to
        256 tokens takes ~4x the batch-1 prefill of the same prompts), at least one of each."""
        groups = world // tp
        pg = max(1, min(groups - 1, round(groups / 4)))
        return cls(world, pg * tp, tp)

    @property
    def n_prefill_groups(self) -> int:
        return self.prefill_gpus // self.tp

    @property
    def n_decode_groups(self) -> int:
        return (self.world - self.prefill_gpus) // self.tp

    def prefill_ranks(self, g: int) -> list[int]:
        return list(range(g * self.tp, (g + 1) * self.tp))

    def decode_ranks(self, j: int) -> list[int]:
        base = self.prefill_gpus + j * self.tp
        return list(range(base, base + self.tp))

    def feeder(self, j: int) -> int:
        return j % self.n_prefill_groups

    def fed_by(self, g: int) -> list[int]:
        return [j for j in range(self.n_decode_groups) if self.feeder(j) == g]

    def role(self, rank: int) -> tuple[str, int, int]:
        """("prefill" | "decode", group index, TP index) of a rank."""
        if rank < self.prefill_gpus:
            return "prefill", rank // self.tp, rank % self.tp
        r = rank - self.prefill_gpus
        return "decode", r // self.tp, r % self.tp

    def describe(self) -> str:
        return (f"{self.n_prefill_groups} prefill group(s) x TP{self.tp} on GPUs 0-{self.prefill_gpus - 1}, "
                f"{self.n_decode_groups} decode group(s) x TP{self.tp} on GPUs "
                f"{self.prefill_gpus}-{self.world - 1}")


@dataclass
class Request:
    rid: int
    prompt: list
    max_new: int
    arrival: float = 0.0     # seconds after the serving start
    group: int = -1          # decode group (set by assign)
    index: int = -1          # position in that group's admission order


def assign(requests: list[Request], split: Split) -> list[Request]:
    """Round-robin over decode groups in arrival order; index = order within the group."""
    counts = [0] * split.n_decode_groups
    for n, r in enumerate(sorted(requests, key=lambda r: (r.arrival, r.rid))):
        r.group = n % split.n_decode_groups
        r.index = counts[r.group]
        counts[r.group] += 1
    return requests


class ByteRing:
    """Sender-side bookkeeping of a FIFO byte ring in the receiver's memory: regions are
    reserved in order, wrap to offset 0 when the tail does not fit, and a region is reused only
    after the receiver released every older region that overlaps it."""

    def __init__(self, size: int):
        self.size = size
        self.live: deque = deque()  # (index, start, end) not yet released, oldest first

    def reserve(self, index: int, nbytes: int, wait_released) -> int:
        nbytes = (nbytes + ALIGN - 1) // ALIGN * ALIGN
        if nbytes > self.size:
            raise ValueError(f"a request needs {nbytes} bytes of staging, the ring holds {self.size}")
        start = self.live[-1][2] if self.live else 0
        if start + nbytes > self.size:
            start = 0
        end = start + nbytes
        while self.live and any(s < end and start < e for _, s, e in self.live):
            wait_released(self.live[0][0])
            self.live.popleft()
        self.live.append((index, start, end))
        return start


def _keys(prefix, j, t, k):
    return f"{prefix}/rdy/{j}/{t}/{k}", f"{prefix}/free/{j}/{t}/{k}"


def make_groups(split: Split):
    """TP process groups of every prefill and decode group (collective: all ranks call it in
    the same order). Returns this rank's group (None when tp == 1)."""
    mine = None
    rank = dist.get_rank()
    for g in range(split.n_prefill_groups):
        ranks = split.prefill_ranks(g)
        pg = dist.new_group(ranks) if split.tp > 1 else None
        if rank in ranks:
            mine = pg
    for j in range(split.n_decode_groups):
        ranks = split.decode_ranks(j)
        pg = dist.new_group(ranks) if split.tp > 1 else None
        if rank in ranks:
            mine = pg
    return mine


def connect_rings(split: Split, ring_bytes: int):
    """Exchanges CUDA-IPC handles of every decode rank's staging ring with its prefill peer, in
    one global order (deadlock-free). Returns (handoffs, local ring tensor or None,
    {decode group: remote address} for a prefill rank)."""
    rank = dist.get_rank()
    handoffs, staging, remotes = [], None, {}
    for j in range(split.n_decode_groups):
        for t in range(split.tp):
            d = split.decode_ranks(j)[t]
            p = split.prefill_ranks(split.feeder(j))[t]
            if rank == d:
                h = KVHandoff(p)
                staging = h.expose(ring_bytes)
                handoffs.append(h)
            elif rank == p:
                h = KVHandoff(d)
                remotes[j] = h.attach()
                handoffs.append(h)
    return handoffs, staging, remotes


class PrefillWorker:
    """One prefill rank: packed prefill of the requests that have arrived, greedy first tokens,
    one gather-pack per request into its decode peer's ring."""

    def __init__(self, engine, split: Split, store, remotes: dict, ring_bytes: int,
                 max_prompt: int, max_tokens: int = PREFILL_TOKENS,
                 max_prompts: int = PREFILL_PROMPTS):
        self.eng, self.split, self.store = engine, split, store
        kind, self.g, self.t = split.role(dist.get_rank())
        assert kind == "prefill"
        self.remotes = remotes
        self.rings = {j: ByteRing(ring_bytes) for j in remotes}
        self.max_tokens, self.max_prompts = max(max_tokens, max_prompt), max_prompts
        m = engine.model
        self.cap = max_prompt
        self.cache = m.allocate_inference_cache(max_prompts, self.cap)
        c0 = self.cache[0]
        self.elem = c0.element_size()
        self.layer_stride = self.cache[1].data_ptr() - c0.data_ptr() if m.n_layer > 1 else 0
        self.row_stride = c0.stride(1) * self.elem
        self.src = torch.tensor([c0.data_ptr() + b * c0.stride(0) * self.elem
                                 for b in range(max_prompts)], dtype=torch.int64,
                                device=engine.device)
        self.first = torch.empty(max_prompts, dtype=torch.long, device=engine.device)
        self.stats: list[dict] = []

    @torch.inference_mode()
    def run(self, requests: list[Request], prefix: str, t0: float, device_ids: dict | None = None):
        """Serves this prefill group's share of `requests` (group and index set) in arrival
        order; `prefix` namespaces the store keys of this run. device_ids optionally maps
        rid -> a device-resident [1, L] id tensor (otherwise ids come from pinned host memory).
        Every pass takes the requests that have arrived, up to max_tokens tokens and
        max_prompts prompts (all TP ranks of the group take the same ones: their decisions
        depend only on arrival times, which they read against the same start)."""
        mine = [r for r in requests if self.split.feeder(r.group) == self.g]
        mine.sort(key=lambda r: (r.arrival, r.rid))
        for ring in self.rings.values():  # the previous run ended with every region consumed
            ring.live.clear()
        m, eng = self.eng.model, self.eng
        dev = eng.device
        n = m.n_layer
        tp = self.split.tp
        i = 0
        while i < len(mine):
            now = time.monotonic() - t0
            if mine[i].arrival > now:
                time.sleep(mine[i].arrival - now)
                now = time.monotonic() - t0
            if tp > 1:
                # The group's ranks must batch the same requests: the first rank's clock decides.
                now = self._agree(now)
            # A pass reserves ring space for all its requests before publishing any of them, so
            # its bytes per ring stay within half the ring: a reservation then only ever waits
            # for regions of earlier, already published passes.
            j, tok, per_ring = i, 0, {}
            while j < len(mine) and j - i < self.max_prompts:
                r = mine[j]
                nb = n * len(r.prompt) * eng.row_bytes + ALIGN
                if j > i and (r.arrival > now or tok + len(r.prompt) > self.max_tokens
                              or per_ring.get(r.group, 0) + nb > self.rings[r.group].size // 2):
                    break
                tok += len(r.prompt)
                per_ring[r.group] = per_ring.get(r.group, 0) + nb
                j += 1
            batch = mine[i:j]
            for r in batch:
                if len(r.prompt) > self.cap:
                    raise ValueError(f"prompt of {len(r.prompt)} tokens exceeds the prefill "
                                     f"capacity {self.cap}")
            start = time.monotonic() - t0
            offs = [self.rings[r.group].reserve(
                r.index, n * len(r.prompt) * eng.row_bytes,
                lambda k, r=r: self.store.wait([_keys(prefix, r.group, self.t, k)[1]]))
                for r in batch]
            lens = [len(r.prompt) for r in batch]
            if device_ids:
                ids = torch.cat([device_ids[r.rid].view(-1) for r in batch])
            else:
                ids = torch.tensor([t for r in batch for t in r.prompt],
                                   dtype=torch.long).pin_memory().to(dev, non_blocking=True)
            live = torch.tensor(lens, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            dst = torch.tensor(offs, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            m.prefill_packed(ids, lens, self.cache, list(range(len(batch))),
                             out=self.first[:len(batch)])
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for b, r in enumerate(batch):
                ops.kv_pack(self.src[b:b + 1], live[b:b + 1], dst[b:b + 1], n, self.layer_stride,
                            self.row_stride, eng.row_bytes, lens[b], self.remotes[r.group])
            e1.record()
            # Every pack has completed (its peer stores have landed) before a key is published.
            torch.cuda.current_stream().synchronize()
            firsts = self.first[:len(batch)].tolist()
            ready = time.monotonic() - t0
            kv_ms = e0.elapsed_time(e1)
            kv_bytes = n * sum(lens) * eng.row_bytes
            for b, r in enumerate(batch):
                self.store.set(_keys(prefix, r.group, self.t, r.index)[0],
                               json.dumps({"tok": firsts[b], "L": lens[b], "off": offs[b]}))
                self.stats.append({"rid": r.rid, "arrival": r.arrival, "start": start,
                                   "ready": ready, "kv_bytes": n * lens[b] * eng.row_bytes,
                                   "kv_ms": kv_ms * lens[b] / sum(lens), "batch": len(batch),
                                   "pass_kv_bytes": kv_bytes, "pass_kv_ms": kv_ms})
            i = j

    def _agree(self, now: float) -> float:
        t = torch.tensor([now], dtype=torch.float64, device=self.eng.device)
        dist.broadcast(t, src=self.split.prefill_ranks(self.g)[0],
                       group=self.eng.model.process_group)
        return float(t.item())


class DecodeWorker:
    """One decode rank: a ContinuousBatcher fed from this rank's staging ring."""

    def __init__(self, engine, split: Split, store, staging: torch.Tensor, slots: int,
                 capacity: int):
        self.eng, self.split, self.store, self.staging = engine, split, store, staging
        kind, self.j, self.t = split.role(dist.get_rank())
        assert kind == "decode"
        self.batcher = ContinuousBatcher(engine, slots, capacity)
        self.stats: list[dict] = []
        self.steps = 0
        self.step_times: list[tuple] = []  # (control s, step s, active slots) per decode step

    @torch.inference_mode()
    def run(self, requests: list[Request], prefix: str, t0: float, poll_s: float = 0.0005):
        """Serves this decode group's requests (admitted in index order); returns
        {rid: generated tokens}."""
        mine = sorted((r for r in requests if r.group == self.j), key=lambda r: r.index)
        pending = deque(mine)
        by_id = {r.rid: r for r in mine}
        tp, leader = self.split.tp, self.t == 0
        b = self.batcher
        done, step = 0, 0
        admitted_at = {}
        while done < len(mine):
            t_loop = time.perf_counter()
            adm = []
            if leader:
                free = len(b.free_slots())
                while pending and free:
                    k = pending[0].index
                    if not self.store.check([_keys(prefix, self.j, t, k)[0] for t in range(tp)]):
                        break
                    adm.append(pending.popleft().rid)
                    free -= 1
                if tp > 1:
                    self.store.set(f"{prefix}/adm/{self.j}/{step}", json.dumps(adm))
            else:
                adm = json.loads(self.store.get(f"{prefix}/adm/{self.j}/{step}"))
            for rid in adm:
                r = by_id[rid]
                rec = json.loads(self.store.get(_keys(prefix, self.j, self.t, r.index)[0]))
                b.admit_packed(rid, self.staging, rec["off"], rec["L"], rec["tok"], r.max_new)
                admitted_at[rid] = time.monotonic() - t0
                if r.max_new == 1:  # finished at its first token
                    done += 1
                    self.stats.append({"rid": rid, "tokens": 1, "done": admitted_at[rid],
                                       "admitted": admitted_at[rid]})
            if b.active():
                t_step = time.perf_counter()
                finished = b.step()
                self.steps += 1
                # Host wall time per decode iteration: control (store, admissions) and the step
                # (graph replay up to the tokens read back).
                self.step_times.append((t_step - t_loop, time.perf_counter() - t_step, b.active()))
            else:
                finished = []
                if adm:
                    torch.cuda.current_stream().synchronize()
                elif leader:
                    time.sleep(poll_s)
            # Every scatter issued above has completed (the step read its tokens back, or the
            # stream was synchronised): release the ring regions.
            for rid in adm:
                self.store.set(_keys(prefix, self.j, self.t, by_id[rid].index)[1], "1")
            now = time.monotonic() - t0
            for rid in finished:
                done += 1
                self.stats.append({"rid": rid, "tokens": len(b.out[rid]), "done": now,
                                   "admitted": admitted_at[rid]})
            step += 1
        return {rid: b.out[rid] for rid in by_id}
