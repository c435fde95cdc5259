"""Pipeline over the local GPUs: one process per GPU, one stage per process.

This replaces the reference's master/worker hand-off (the hidden state
serialised to bytes and sent over TCP, spm/message.rs:147-165 and 366-408,
worker loop spm/worker.rs:645-765, Client::forward_batch spm/client.rs:389-452)
with device-to-device sends over NVLink: stage s sends the bf16/f16 hidden
state [rows, hidden] of each micro-batch to stage s+1, and the last stage
sends each sequence's next token id (int32) back to stage 0, which embeds it
for the next step.  Layers are split by the stage planner (planner.py).

Schedule (every stage, micro-batches b = 0..B-1 of step t, m = t*B + b):
    stage 0:    input = token of m-B from the last stage (t > 0) or the prompt's
                first token (t = 0)
    stage s>0:  input = hidden of m from stage s-1
    compute     (embedding on stage 0, layers, head + argmax on the last stage)
    stage s<P-1: hidden of m -> stage s+1;  last stage: token of m -> stage 0
With B >= P micro-batches every stage is busy in the steady state.  Sends are
asynchronous (a send buffer is reused only after its previous send finished)
and each stage pair has its own channel, so the token ring back to stage 0
cannot block the forward chain.

Vocabulary-parallel head (Pipeline(..., head_channel=, head_rows=)): every
stage holds a share of the output head's rows; the last stage sends each
micro-batch's final hidden state to the stages with rows (on a side stream,
so the forward chain does not wait for it), each computes the greedy keys of
its rows (final norm + GEMV + argmax, dial_decoder_head_shard) and sends them
to stage 0, which merges them into the token (dial_head_merge) -- no stage
reads the whole head, and the token ring carries 8-byte keys instead of the
token.  This is the reference's output head split by vocabulary rows (its
head runs on the last worker, worker_gguf.rs:342-386, qwen3_vl.rs:2420-2451).

The communication is a `Channel` object: NcclChannel (the C ABI's NCCL stage
communicators, dial_stage_comm_*, over NVLink between GPUs) or TorchChannel
(torch.distributed point-to-point; gloo for the CPU tests).  The compute of a
stage is a `StageCompute` object; ModelStageCompute runs a model.Stage.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional, Sequence


def _torch():
    import torch  # noqa: PLC0415
    return torch


# ------------------------------------------------------------------ channels
def pipeline_links(P: int) -> List[tuple]:
    """The hand-off links: stage s -> s+1, and the token ring P-1 -> 0."""
    return [(s, s + 1) for s in range(P - 1)] + ([(P - 1, 0)] if P > 1 else [])


def head_links(P: int, rows: Sequence) -> List[tuple]:
    """The vocabulary-parallel head's links, in their global set-up order: the
    last stage's final hidden state to every other stage with head rows, then
    each stage's greedy keys to stage 0 (the last stage's keys reuse its link
    to stage 0)."""
    out = [(P - 1, s) for s in range(P - 1) if rows[s]]
    out += [(s, 0) for s in range(1, P - 1) if rows[s]]
    if rows[P - 1] and (P - 1, 0) not in out:
        out.append((P - 1, 0))
    return out


class TorchChannel:
    """Point-to-point sends over torch.distributed, one process group per link:
    fwd[s] carries stage s -> s+1, `ring` carries the last stage -> stage 0.
    Separate groups are separate NCCL communicators with their own streams, so
    a blocked send on one link never holds up another link's operations.
    Every rank creates every group, in the same order (a torch requirement)."""

    def __init__(self, world: Optional[int] = None, links: Optional[List[tuple]] = None):
        import torch.distributed as dist  # noqa: PLC0415
        self.dist = dist
        self.rank = dist.get_rank()
        P = world if world is not None else dist.get_world_size()
        self.P = P
        self.links = list(links) if links is not None else pipeline_links(P)
        self.groups = [dist.new_group(sorted({a, b})) for a, b in self.links]

    def _group(self, a: int, b: int):  # link a -> b
        if (a, b) in self.links:
            return self.groups[self.links.index((a, b))]
        raise ValueError(f"no pipeline link {a} -> {b}")

    def isend(self, t, dst: int):
        return self.dist.isend(t, dst, group=self._group(self.rank, dst))

    def irecv(self, t, src: int):
        return self.dist.irecv(t, src, group=self._group(src, self.rank))


class _Done:
    """A transfer enqueued on a link's stream: wait() orders the caller's
    current stream after it (the host does not block)."""

    def __init__(self, event):
        self.event = event

    def wait(self):
        _torch().cuda.current_stream().wait_event(self.event)


class NcclChannel:
    """The pipeline's links over the C ABI's NCCL stage communicators
    (dial_stage_comm_*): link s carries stage s -> s+1, the last link the token
    ring from stage P-1 to stage 0.  Each link is a two-rank communicator (link
    rank 0 = its sender) with its own CUDA stream, so a transfer waiting on one
    link never holds up another.  Each link's sender makes the clique id; the
    ids are shared with one all_gather_object on the default torch.distributed
    group (bootstrap only: no tensor crosses it).  Every rank initialises its
    links in the global link order, so no two ranks wait on each other's
    initialisation in a cycle; every host wait is bounded by `timeout_s`."""

    def __init__(self, rank: int, world: int, timeout_s: float = 60.0,
                 links: Optional[List[tuple]] = None):
        import ctypes  # noqa: PLC0415

        import torch.distributed as dist  # noqa: PLC0415

        from . import ID_BYTES, check, lib  # noqa: PLC0415
        torch = _torch()
        self.rank, self.P, self.L = rank, world, lib()
        self.links = list(links) if links is not None else pipeline_links(world)
        mine = {}
        for i, (a, _) in enumerate(self.links):
            if a == rank:
                buf = (ctypes.c_uint8 * ID_BYTES)()
                check(self.L.dial_stage_comm_unique_id(buf), "dial_stage_comm_unique_id")
                mine[i] = bytes(buf)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        ids = {}
        for d in gathered:
            ids.update(d)
        dev = torch.cuda.current_device()
        self.comms = {}  # link index -> (communicator, stream, my rank in the link)
        for i, (a, b) in enumerate(self.links):
            if rank not in (a, b):
                continue
            lr = 0 if rank == a else 1
            comm = ctypes.c_void_p()
            idbuf = (ctypes.c_uint8 * ID_BYTES).from_buffer_copy(ids[i])
            check(self.L.dial_stage_comm_init(idbuf, lr, 2, dev, timeout_s, ctypes.byref(comm)),
                  f"dial_stage_comm_init(link {a}->{b})")
            self.comms[i] = (comm, torch.cuda.Stream(device=dev), lr)

    def _link(self, a: int, b: int) -> int:
        return self.links.index((a, b))

    def _op(self, fn, t, link: int, where: str):
        from . import check  # noqa: PLC0415
        torch = _torch()
        comm, stream, lr = self.comms[link]
        stream.wait_stream(torch.cuda.current_stream())  # the buffer's producers (or readers)
        check(fn(comm, t.data_ptr(), t.numel() * t.element_size(), 1 - lr, stream.cuda_stream), where)
        t.record_stream(stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        return _Done(ev)

    def isend(self, t, dst: int):
        return self._op(self.L.dial_stage_comm_send, t, self._link(self.rank, dst), "dial_stage_comm_send")

    def irecv(self, t, src: int):
        return self._op(self.L.dial_stage_comm_recv, t, self._link(src, self.rank), "dial_stage_comm_recv")

    def close(self) -> None:
        """Waits (bounded) for each link's transfers, then frees its communicator."""
        from . import check  # noqa: PLC0415
        for comm, stream, _ in self.comms.values():
            check(self.L.dial_stage_comm_wait(comm, stream.cuda_stream), "dial_stage_comm_wait")
            check(self.L.dial_stage_comm_destroy(comm), "dial_stage_comm_destroy")
        self.comms = {}


def init_distributed(backend: str = "nccl", timeout_s: float = 120.0):
    """rank, local_rank, world from the torchrun environment; short timeout so
    that ranks waiting on a dead peer end with an error."""
    import torch.distributed as dist  # noqa: PLC0415
    torch = _torch()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, local, world


# ------------------------------------------------------------------ stage compute
class StageCompute:
    """What one stage does to micro-batch b.  Buffers are fixed per micro-batch.
    For prefill: prefill_buffer(T) is the [T, hidden] hand-off buffer and
    prefill_run(b, ids) runs stage 0's embedding of `ids`, the layers, and the
    last stage's head on the last row (the first token, into token_buffer(b))."""

    first: bool
    last: bool

    def hidden_buffer(self, b: int):  # [rows, hidden] in the activation dtype
        raise NotImplementedError

    def token_buffer(self, b: int):  # int32 [rows]
        raise NotImplementedError

    def run(self, b: int) -> None:
        """Stage 0 embeds token_buffer(b); every stage runs its layers on
        hidden_buffer(b); the last stage writes the next token to token_buffer(b)."""
        raise NotImplementedError

    def advance(self, b: int) -> None:
        """Moves micro-batch b to its next position (after its step)."""


class ModelStageCompute(StageCompute):
    """A model.Stage driving n_mb micro-batches of `mb_size` sequences each
    (micro-batch b holds KV slots b*mb_size .. b*mb_size + mb_size - 1), each
    step captured once as a CUDA graph per micro-batch."""

    def __init__(self, stage, n_mb: int, prompt_len: int, use_graphs: bool = True, mb_size: int = 1,
                 vocab_head_stages: int = 0):
        """vocab_head_stages = P: the head is vocabulary-parallel over P stages
        (the stage holds rows stage.head_rows; the last stage runs no head)."""
        torch = _torch()
        self.st = stage
        self.first, self.last = stage.first == 0, stage.last == stage.cfg.n_layers
        self.n_mb, self.mb_size = n_mb, mb_size
        dev, dt, H, R = stage.device, stage.dt, stage.cfg.hidden, mb_size
        self.hidden = [torch.zeros((R, H), device=dev, dtype=dt) for _ in range(n_mb)]
        self.tokens = [torch.zeros(R, device=dev, dtype=torch.int32) for _ in range(n_mb)]
        self.vocab_head = vocab_head_stages > 0
        if self.vocab_head:
            P = vocab_head_stages
            self.head_in = [torch.zeros((R, H), device=dev, dtype=dt) for _ in range(n_mb)]
            # stage 0 gathers every stage's keys ([P, R], its own in row 0)
            self.keys = [torch.zeros((P if self.first else 1, R), device=dev, dtype=torch.int64)
                         for _ in range(n_mb)]
        self.pos = [torch.full((R,), prompt_len, device=dev, dtype=torch.int32) for _ in range(n_mb)]
        self.slot = [torch.arange(b * R, (b + 1) * R, device=dev, dtype=torch.int32) for b in range(n_mb)]
        self.use_graphs = use_graphs
        self.graphs: List = [None] * n_mb

    def hidden_buffer(self, b):
        return self.hidden[b]

    def token_buffer(self, b):
        return self.tokens[b]

    def _eager(self, b):
        st = self.st
        if self.first:
            st.embed_tokens(self.tokens[b], self.hidden[b])
        st.layers_forward(self.hidden[b], self.pos[b], self.slot[b], st.max_seq)
        if self.last and not self.vocab_head:
            st.head_forward(self.hidden[b], self.tokens[b])

    # vocabulary-parallel head
    def head_input(self, b):  # where the last stage's final hidden state arrives
        return self.hidden[b] if self.last else self.head_in[b]

    def head_keys(self, b):  # this stage's keys [R]
        return self.keys[b][0]

    def gathered_keys(self, b, s):  # stage 0: the row of stage s's keys
        return self.keys[b][s]

    def run_head_shard(self, b):
        self.st.head_shard_forward(self.head_input(b), self.head_keys(b))

    def merge(self, b):
        from .model import head_merge  # noqa: PLC0415
        head_merge(self.keys[b], self.tokens[b])

    def capture(self) -> None:
        """Captures one graph per micro-batch (its positions advance in place)."""
        if not self.use_graphs:
            return
        torch = _torch()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for b in range(self.n_mb):
                self._eager(b)  # warm: workspaces, kernel attributes
        torch.cuda.synchronize()
        for b in range(self.n_mb):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                self._eager(b)
            self.graphs[b] = g
        torch.cuda.synchronize()

    def run(self, b):
        if self.graphs[b] is not None:
            self.graphs[b].replay()
        else:
            self._eager(b)

    def advance(self, b):
        self.pos[b].add_(1)

    def reset_positions(self, prompt_len: int) -> None:
        for p in self.pos:
            p.fill_(prompt_len)

    # prefill: one sequence (KV slot b) of T prompt tokens per micro-batch
    def prefill_buffer(self, T: int):
        torch = _torch()
        if getattr(self, "_pbuf", None) is None or self._pbuf.shape[0] != T:
            self._pbuf = torch.empty((T, self.st.cfg.hidden), device=self.st.device, dtype=self.st.dt)
            self._ppos = torch.arange(T, device=self.st.device, dtype=torch.int32)
            self._plast = torch.tensor([T - 1], device=self.st.device, dtype=torch.int32)
        return self._pbuf

    def prefill_run(self, b: int, ids=None, i: int = 0) -> None:
        """Prefills sequence i of micro-batch b (KV slot b*mb_size + i); stage 0
        embeds its prompt `ids` [T]."""
        torch = _torch()
        st, h = self.st, self._pbuf
        T = h.shape[0]
        seq = b * self.mb_size + i
        if self.first:
            st.embed_tokens(ids, h)
        st.layers_forward(h, self._ppos, torch.full((T,), seq, device=st.device, dtype=torch.int32), T)
        if self.last and self.vocab_head:  # the head runs on every stage (Pipeline._head_exchange)
            self.hidden[b][i].copy_(h[T - 1])
        elif self.last:
            st.head_forward(h, self.tokens[b][i:i + 1], row_index=self._plast)


# ------------------------------------------------------------------ the schedule
class Pipeline:
    """Stage `rank` of a `world`-stage pipeline over n_mb micro-batches."""

    def __init__(self, rank: int, world: int, compute: StageCompute, channel, n_mb: int,
                 head_channel=None, head_rows: Optional[Sequence] = None):
        """head_rows (per stage, the number of head rows it holds) with
        head_channel (links head_links(world, head_rows)): the head is
        vocabulary-parallel; otherwise it runs on the last stage."""
        if world > 1 and n_mb < world:
            raise ValueError(f"{n_mb} micro-batches cannot keep {world} stages busy")
        self.rank, self.world, self.c, self.ch, self.n_mb = rank, world, compute, channel, n_mb
        self.vocab = head_rows is not None and world > 1
        self.hch, self.rows = head_channel, list(head_rows) if head_rows is not None else None
        if self.vocab and (head_channel is None or not getattr(compute, "vocab_head", False)):
            raise ValueError("a vocabulary-parallel head needs head_channel and a vocab-head compute")
        self.head_pending = [[] for _ in range(n_mb)]  # head sends that read this micro-batch's buffers
        self.merged = [None] * n_mb  # stage 0: event of each micro-batch's merged token
        self._hs = None  # the head's side stream
        self.pending = [None] * n_mb  # last send of each micro-batch's output buffer
        self.t = 0  # decode steps since the last prefill
        self.host_io = None  # (host_in, host_out): pinned int32 token copies for host_io steps
        self._connected = False  # decode-sized transfers made on every link (_connect)
        self._prefill_connected = set()  # prompt lengths whose hand-off sizes were exchanged

    def _wait_send(self, b):
        if self.pending[b] is not None:
            self.pending[b].wait()
            self.pending[b] = None

    def _connect(self, fwd, ring) -> None:
        """One matched transfer per link, in link order (0 -> 1, ..., P-2 -> P-1,
        then P-1 -> 0), of tensors shaped like that link's traffic.

        NCCL sets up a peer connection on the host at the first transfer between
        two ranks, and that call returns only once the peer makes its matching
        call.  Without this exchange the ring's first send (the last stage's
        first prefill tokens) blocks the last stage's host until stage 0 reaches
        its first receive on the ring, after its whole prefill loop; stage 0's
        host meanwhile blocks in a kernel launch once its stream, held up by
        a forward send that the last stage has not received yet, has a full
        launch queue.  Here every rank meets its links in one order, so the
        set-ups form a chain and cannot wait in a cycle."""
        r, P, ch = self.rank, self.world, self.ch
        for s in range(P - 1):
            if r == s:
                ch.isend(fwd, s + 1).wait()
            elif r == s + 1:
                ch.irecv(fwd, s).wait()
        if r == P - 1:
            ch.isend(ring, 0).wait()
        elif r == 0:
            ch.irecv(ring, P - 1).wait()

    def _connect_head(self) -> None:
        """One matched transfer per head link and message kind, in head_links
        order (as _connect): the final hidden state on the last stage's links,
        keys on the links into stage 0."""
        r, P, c = self.rank, self.world, self.c
        h, k = c.hidden_buffer(0).clone(), c.head_keys(0).clone()
        for a, b in head_links(P, self.rows):
            kinds = ([h] if a == P - 1 and self.rows[b] else []) + ([k] if b == 0 and self.rows[a] else [])
            for t in kinds:
                if r == a:
                    self.hch.isend(t, b).wait()
                elif r == b:
                    self.hch.irecv(t, a).wait()

    def _connect_steps(self) -> None:
        if self.world > 1 and not self._connected:
            c = self.c
            self._connect(c.hidden_buffer(0).clone(), c.token_buffer(0).clone())
            if self.vocab:
                self._connect_head()
            self._connected = True

    def _wait_merged(self, b) -> None:  # stage 0: b's tokens are merged
        if self.merged[b] is not None:
            _torch().cuda.current_stream().wait_event(self.merged[b])

    def _wait_head(self, b) -> None:
        for d in self.head_pending[b]:
            d.wait()
        self.head_pending[b] = []

    def _head_exchange(self, b) -> None:
        """The vocabulary-parallel head for micro-batch b (every stage, after
        its compute of b): on the side stream, the last stage sends the final
        hidden state to the stages with rows, each computes its keys and sends
        them to stage 0, and stage 0 merges them into b's tokens."""
        import contextlib  # noqa: PLC0415
        torch = _torch()
        r, P, c, hch = self.rank, self.world, self.c, self.hch
        cuda = torch.cuda.is_available()  # (the CPU tests run it synchronously over gloo)
        if cuda and self._hs is None:
            self._hs = torch.cuda.Stream()
        hs = self._hs
        if cuda:
            hs.wait_stream(torch.cuda.current_stream())  # b's compute on this stage
        with torch.cuda.stream(hs) if cuda else contextlib.nullcontext():
            self._wait_head(b)  # the buffers of b's previous exchange are free again
            sends = []
            if r == P - 1:
                sends += [hch.isend(c.hidden_buffer(b), s) for s in range(P - 1) if self.rows[s]]
            elif self.rows[r]:
                hch.irecv(c.head_input(b), P - 1).wait()
            if self.rows[r]:
                c.run_head_shard(b)
                if r != 0:
                    sends.append(hch.isend(c.head_keys(b), 0))
            self.head_pending[b] = sends
            if r == 0:
                for s in range(1, P):
                    if self.rows[s]:
                        hch.irecv(c.gathered_keys(b, s), s).wait()
                c.merge(b)
                ev = None
                if cuda:
                    ev = torch.cuda.Event()
                    ev.record(hs)
                self.merged[b] = ev

    def steps(self, n_steps: int, host_io: bool = False) -> None:
        """n_steps decode steps: every micro-batch advances one token per step.
        The last stage sends every token back to stage 0 (which embeds it at the
        next step); finish() takes in the last step's tokens.  With host_io the
        tokens also pass through pinned host memory as in a serving loop: stage 0
        reads each token it receives back to the host and embeds the host copy
        (one host synchronisation per micro-batch), and the last stage copies the
        step's tokens to the host and synchronises at the end of the step."""
        torch = _torch() if host_io else None
        r, P, B, c, ch = self.rank, self.world, self.n_mb, self.c, self.ch
        self._connect_steps()
        if host_io and self.host_io is None:
            n = [c.token_buffer(b).numel() for b in range(B)]  # one token per row
            self.host_io = ([torch.zeros(n[b], dtype=torch.int32).pin_memory() for b in range(B)],
                            [torch.zeros(n[b], dtype=torch.int32).pin_memory() for b in range(B)])
        for _ in range(n_steps):
            for b in range(B):
                tok = c.token_buffer(b)
                if P > 1:
                    self._wait_send(b)  # the buffer is an input of this micro-batch again
                    if self.vocab:
                        self._wait_head(b)
                    if r == 0:
                        if self.vocab:
                            self._wait_merged(b)
                        elif self.t > 0:
                            ch.irecv(tok, P - 1).wait()
                    else:
                        ch.irecv(c.hidden_buffer(b), r - 1).wait()
                if host_io and r == 0:
                    hin = self.host_io[0][b]
                    hin.copy_(tok, non_blocking=True)
                    torch.cuda.current_stream().synchronize()
                    tok.copy_(hin, non_blocking=True)
                c.run(b)
                c.advance(b)
                if host_io and r == P - 1 and not self.vocab:
                    self.host_io[1][b].copy_(tok, non_blocking=True)
                if P > 1:
                    if r < P - 1:
                        self.pending[b] = ch.isend(c.hidden_buffer(b), r + 1)
                    elif not self.vocab:
                        self.pending[b] = ch.isend(tok, 0)
                    if self.vocab:
                        self._head_exchange(b)
            if host_io and r == P - 1 and not self.vocab:
                torch.cuda.current_stream().synchronize()
            self.t += 1

    def finish(self) -> None:
        """Ends a decode run: stage 0 takes in the last step's tokens (its token
        buffers then hold every sequence's latest token), every stage waits for
        its sends."""
        if self.world > 1 and self.rank == 0 and self.t > 0:
            for b in range(self.n_mb):
                if self.vocab:
                    self._wait_merged(b)
                else:
                    self.ch.irecv(self.c.token_buffer(b), self.world - 1).wait()
        self.drain()
        self.t = 0

    def host_tokens(self):
        """The last host_io step's tokens (last stage)."""
        return [int(x) for t in self.host_io[1] for x in t.tolist()] if self.host_io else None

    def drain(self) -> None:
        for b in range(self.n_mb):
            self._wait_send(b)
            self._wait_head(b)

    def prefill(self, prompts: Optional[Sequence] = None, prompt_len: int = 0) -> None:
        """Prefills every sequence (stage 0 holds the prompts, one per sequence,
        micro-batch-major); the first generated tokens end up in stage 0's token
        buffers.  The [T, hidden] hand-off reuses one buffer per stage, so each
        send completes before the next sequence overwrites it."""
        r, P, B, c, ch = self.rank, self.world, self.n_mb, self.c, self.ch
        R = getattr(c, "mb_size", 1)
        T = len(prompts[0]) if prompts is not None else prompt_len
        buf = c.prefill_buffer(T)
        if P > 1 and T not in self._prefill_connected:
            # once per hand-off size: NCCL may open further connections for a
            # larger message the first time one crosses a link
            self._connect(buf, c.token_buffer(0).clone())
            self._connect_steps()
            self._prefill_connected.add(T)
        for b in range(B):
            for i in range(R):
                if r > 0:
                    ch.irecv(buf, r - 1).wait()
                if R == 1:
                    c.prefill_run(b, prompts[b] if r == 0 else None)
                else:
                    c.prefill_run(b, prompts[b * R + i] if r == 0 else None, i)
                if r < P - 1:
                    ch.isend(buf, r + 1).wait()
            if self.vocab:
                self._head_exchange(b)
            elif r == P - 1 and P > 1:
                self.pending[b] = ch.isend(c.token_buffer(b), 0)
        if P > 1 and r == 0:
            for b in range(B):
                if self.vocab:
                    self._wait_merged(b)
                else:
                    ch.irecv(c.token_buffer(b), P - 1).wait()
        self.drain()
        self.t = 0


def even_split(n_layers: int, n_stages: int) -> List[range]:
    """Contiguous, as even as possible (the first stages get the extra layers)."""
    q, rem = divmod(n_layers, n_stages)
    out, a = [], 0
    for s in range(n_stages):
        n = q + (1 if s < rem else 0)
        out.append(range(a, a + n))
        a += n
    return out


def stage_layers(n_layers: int, world: int, head_layers: float = 3.2,
                 method: str = "planner") -> List[range]:
    """Layer ranges per stage: the planner's bottleneck-balanced split (the head
    counted as `head_layers` layers on the last stage) or an even split."""
    if world == 1:
        return [range(0, n_layers)]
    if method == "even":
        return even_split(n_layers, world)
    from .planner import local_gpu_plan  # noqa: PLC0415
    return local_gpu_plan(n_layers, world, head_layers=head_layers, link_latency_ms=0.0)
