"""Pipeline schedule on the CPU: world-size 2, 3 and 4 gloo ranks, a stand-in for
the stage compute, checked against the same chain run in one process, with
micro-batches of one and of several sequences, and over a channel that models
NCCL's blocking link set-up.  Also the failure path: a rank that never joins
makes its peers fail within the process-group timeout instead of hanging."""
import os
import socket
import sys

import pytest

import torch
import torch.multiprocessing as mp

H, V = 8, 97


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeCompute:
    """Stage r of `world`: embedding (stage 0), a per-stage affine map, and a
    token from the hidden state (last stage) -- deterministic f32 arithmetic."""

    def __init__(self, r, world, n_mb):
        self.r, self.world = r, world
        self.first, self.last = r == 0, r == world - 1
        self.hidden = [torch.zeros(1, H) for _ in range(n_mb)]
        self.tokens = [torch.zeros(1, dtype=torch.int32) for _ in range(n_mb)]
        self.pos = [0] * n_mb

    @staticmethod
    def embed(tok):
        return (tok.float() + 1.0) * torch.arange(1, H + 1, dtype=torch.float32) / H

    def layers(self, h, pos):
        return h * 0.75 + 0.125 * (self.r + 1) + 0.01 * pos

    @staticmethod
    def sample(h):
        return torch.tensor([int(h.sum().item() * 1000) % V], dtype=torch.int32)

    def hidden_buffer(self, b):
        return self.hidden[b]

    def token_buffer(self, b):
        return self.tokens[b]

    def run(self, b):
        if self.first:
            self.hidden[b].copy_(self.embed(self.tokens[b]).view(1, H))
        self.hidden[b].copy_(self.layers(self.hidden[b], self.pos[b]))
        if self.last:
            self.tokens[b].copy_(self.sample(self.hidden[b]))

    def advance(self, b):
        self.pos[b] += 1

    def prefill_buffer(self, T):
        self.pbuf = torch.zeros(T, H)
        return self.pbuf

    def prefill_run(self, b, ids=None):
        if self.first:
            self.pbuf.copy_(torch.stack([self.embed(torch.tensor(i)) for i in ids]))
        self.pbuf.copy_(self.layers(self.pbuf, -1))
        if self.last:
            self.tokens[b].copy_(self.sample(self.pbuf[-1]))


class FakeComputeRows(FakeCompute):
    """The same stages with micro-batches of R sequences (rows): each row its own
    sequence, prefilled one sequence at a time (prefill_run's third argument)."""

    def __init__(self, r, world, n_mb, R):
        super().__init__(r, world, n_mb)
        self.mb_size = R
        self.hidden = [torch.zeros(R, H) for _ in range(n_mb)]
        self.tokens = [torch.zeros(R, dtype=torch.int32) for _ in range(n_mb)]

    def run(self, b):
        for i in range(self.mb_size):
            if self.first:
                self.hidden[b][i].copy_(self.embed(self.tokens[b][i]))
            self.hidden[b][i].copy_(self.layers(self.hidden[b][i], self.pos[b]))
            if self.last:
                self.tokens[b][i] = self.sample(self.hidden[b][i])[0]

    def prefill_run(self, b, ids=None, i=0):
        if self.first:
            self.pbuf.copy_(torch.stack([self.embed(torch.tensor(k)) for k in ids]))
        self.pbuf.copy_(self.layers(self.pbuf, -1))
        if self.last:
            self.tokens[b][i] = self.sample(self.pbuf[-1])[0]


def reference(world, n_mb, prompts, steps):
    """The same chain, every stage in one process."""
    stages = [FakeCompute(r, world, n_mb) for r in range(world)]
    out = []
    for b in range(n_mb):
        h = torch.stack([FakeCompute.embed(torch.tensor(i)) for i in prompts[b]])
        for s in stages:
            h = s.layers(h, -1)
        tok = FakeCompute.sample(h[-1])
        seq = [int(tok)]
        for t in range(steps):
            h = FakeCompute.embed(tok).view(1, H)
            for s in stages:
                h = s.layers(h, t)
            tok = FakeCompute.sample(h)
            seq.append(int(tok))
        out.append(seq)
    return out


def _worker(rank, world, port, n_mb, prompts, steps, result_dir, R=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.pipeline import Pipeline, TorchChannel, init_distributed
    init_distributed("gloo", timeout_s=30)
    c = FakeCompute(rank, world, n_mb) if R == 1 else FakeComputeRows(rank, world, n_mb, R)
    p = Pipeline(rank, world, c, TorchChannel(), n_mb)
    p.prefill(prompts if rank == 0 else None, prompt_len=len(prompts[0]))
    firsts = [int(v) for t in c.tokens for v in t.reshape(-1)]
    # two calls of one run, as the benchmark does (warm-up, then timed steps)
    p.steps(2)
    p.steps(steps - 2)
    last = [int(v) for t in c.tokens for v in t.reshape(-1)]
    p.finish()
    torch.save({"firsts": firsts, "last": last,
                "after_finish": [int(v) for t in c.tokens for v in t.reshape(-1)]},
               os.path.join(result_dir, f"r{rank}.pt"))
    import torch.distributed as dist
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_matches_single_process_chain(world, tmp_path):
    n_mb, steps = 3, 5
    prompts = [[(7 * b + 3 * i) % V for i in range(4)] for b in range(n_mb)]
    mp.start_processes(_worker, args=(world, _free_port(), n_mb, prompts, steps, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    ref = reference(world, n_mb, prompts, steps)
    r0 = torch.load(tmp_path / "r0.pt")
    rl = torch.load(tmp_path / f"r{world - 1}.pt")
    assert r0["firsts"] == [seq[0] for seq in ref]          # prefill tokens reached stage 0
    assert rl["last"] == [seq[-1] for seq in ref]           # last step's tokens on the last stage
    assert r0["after_finish"] == [seq[-1] for seq in ref]   # finish() hands them to stage 0


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_micro_batches_of_several_sequences(world, tmp_path):
    """Micro-batches of R = 2 sequences: prefill walks every sequence of a micro-batch
    before the last stage hands that micro-batch's tokens back to stage 0."""
    n_mb, R, steps = 3, 2, 5
    prompts = [[(5 * s + 3 * i + 1) % V for i in range(4)] for s in range(n_mb * R)]
    mp.start_processes(_worker, args=(world, _free_port(), n_mb, prompts, steps, str(tmp_path), R),
                       nprocs=world, join=True, start_method="spawn")
    ref = reference(world, n_mb * R, prompts, steps)
    r0 = torch.load(tmp_path / "r0.pt")
    rl = torch.load(tmp_path / f"r{world - 1}.pt")
    assert r0["firsts"] == [seq[0] for seq in ref]
    assert rl["last"] == [seq[-1] for seq in ref]
    assert r0["after_finish"] == [seq[-1] for seq in ref]


class RendezvousChannel:
    """TorchChannel with two traits of NCCL on GPUs that gloo lacks.  (1) The
    first transfer on a link returns only once the peer has made its own first
    call on that link (NCCL sets up peer connections on the host that way).
    (2) On a forward link, a sender's host blocks while `depth` of its sends
    are not yet received: the prefill makes the compute stream wait on each
    forward send, so an unreceived send holds the stream and the host's later
    launches fill its queue.  The ring's token sends are never waited on by the
    compute stream during prefill (and small NCCL sends finish into the peer's
    buffer), so they do not block the host."""

    def __init__(self, store, rank, world, depth=2, timeout_s=8.0):
        from dial_cuda.pipeline import TorchChannel
        self.inner = TorchChannel(world)
        self.store, self.rank, self.depth, self.timeout_s = store, rank, depth, timeout_s
        self.seen, self.sent, self.got = set(), {}, {}

    def _wait_until(self, cond, what):
        import time
        t0 = time.time()
        while not cond():
            if time.time() - t0 > self.timeout_s:
                raise TimeoutError(what)
            time.sleep(0.002)

    def _first(self, a, b):
        if (a, b) in self.seen:
            return
        self.seen.add((a, b))
        self.store.add(f"link{a}-{b}", 1)
        self._wait_until(lambda: self.store.add(f"link{a}-{b}", 0) >= 2, f"set-up of link {a}->{b}")

    def isend(self, t, dst):
        link = (self.rank, dst)
        self._first(*link)
        if dst == self.rank + 1:
            n = self.sent.get(link, 0)
            key = f"recv{link[0]}-{link[1]}"
            self._wait_until(lambda: self.store.add(key, 0) > n - self.depth, f"send queue of {link}")
            self.sent[link] = n + 1
        return self.inner.isend(t, dst)

    def irecv(self, t, src):
        link = (src, self.rank)
        self._first(*link)
        inner, store = self.inner.irecv(t, src), self.store

        class Done:
            def wait(self_):
                inner.wait()
                store.add(f"recv{link[0]}-{link[1]}", 1)
        return Done()


def _rendezvous_worker(rank, world, port, n_mb, R, prompts, steps, result_dir, skip_connect):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    import torch.distributed as dist
    from dial_cuda.pipeline import Pipeline, init_distributed
    init_distributed("gloo", timeout_s=30)
    store = dist.distributed_c10d._get_default_store()
    c = FakeComputeRows(rank, world, n_mb, R)
    p = Pipeline(rank, world, c, RendezvousChannel(store, rank, world), n_mb)
    if skip_connect:  # the schedule without its link set-up exchange
        p._connect = lambda fwd, ring: None
        p._connected = True
    try:
        p.prefill(prompts if rank == 0 else None, prompt_len=len(prompts[0]))
        p.steps(steps)
        p.finish()
        out = {"ok": True, "tokens": [int(v) for t in c.tokens for v in t.reshape(-1)]}
    except (TimeoutError, RuntimeError) as e:  # gave up, or the peer that gave up left
        out = {"ok": False, "where": str(e)}
    torch.save(out, os.path.join(result_dir, f"rv{rank}.pt"))
    os._exit(0)  # a stuck peer's transfers may still be posted


@pytest.mark.parametrize("world,skip_connect", [(2, False), (2, True), (4, False), (8, False)])
def test_pipeline_link_set_up_cannot_deadlock(world, skip_connect, tmp_path):
    """Two to eight stages, micro-batches of 2 sequences, a channel with NCCL's
    blocking link set-up and bounded send queue: the pipeline finishes and
    matches the single-process chain; without the set-up exchange two stages
    deadlock in prefill (the last stage waits on the ring's set-up, stage 0 on
    its full queue)."""
    n_mb, R, steps = max(3, world), 2, 4
    prompts = [[(11 * s + 5 * i + 2) % V for i in range(3)] for s in range(n_mb * R)]
    mp.start_processes(_rendezvous_worker,
                       args=(world, _free_port(), n_mb, R, prompts, steps, str(tmp_path), skip_connect),
                       nprocs=world, join=True, start_method="spawn")
    outs = [torch.load(tmp_path / f"rv{r}.pt") for r in range(world)]
    if skip_connect:
        assert not outs[1]["ok"] and "set-up of link 1->0" in outs[1]["where"], outs
        return
    assert all(o["ok"] for o in outs), outs
    ref = reference(world, n_mb * R, prompts, steps)
    assert outs[0]["tokens"] == [seq[-1] for seq in ref]


def test_pipeline_rejects_too_few_micro_batches():
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.pipeline import Pipeline
    with pytest.raises(ValueError):
        Pipeline(0, 4, FakeCompute(0, 4, 2), None, 2)


def _lonely(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.pipeline import init_distributed
    try:
        init_distributed("gloo", timeout_s=3)
        msg = "joined"
    except Exception as e:  # the peer never joins: rendezvous times out
        msg = type(e).__name__
    with open(os.path.join(result_dir, f"lonely{rank}.txt"), "w") as f:
        f.write(msg)


def test_missing_peer_fails_within_the_timeout(tmp_path):
    """Rank 0 of a 2-rank group whose rank 1 never starts: it must give up."""
    mp.start_processes(_lonely, args=(2, _free_port(), str(tmp_path)), nprocs=1, join=True,
                       start_method="spawn")
    assert (tmp_path / "lonely0.txt").read_text() != "joined"


# ------------------------------------------------------------------ vocabulary-parallel head
class FakeVocabCompute(FakeComputeRows):
    """The same stages with the head split by vocabulary rows: stage s holds
    rows [v0, v1) of a stand-in head whose logit for id v peaks at
    FakeCompute.sample(h) (so the merged token must equal the single-process
    chain's), and produces greedy keys as dial_decoder_head_shard does
    (value << 32 | 0xFFFFFFFF - id; the largest key is the first maximum)."""

    def __init__(self, r, world, n_mb, R, span):
        super().__init__(r, world, n_mb, R)
        self.vocab_head = True
        self.v0, self.v1 = span
        self.head_in = [torch.zeros(R, H) for _ in range(n_mb)]
        self.keys = [torch.zeros((world if r == 0 else 1, R), dtype=torch.int64) for _ in range(n_mb)]

    def run(self, b):
        for i in range(self.mb_size):
            if self.first:
                self.hidden[b][i].copy_(self.embed(self.tokens[b][i]))
            self.hidden[b][i].copy_(self.layers(self.hidden[b][i], self.pos[b]))

    def prefill_run(self, b, ids=None, i=0):
        if self.first:
            self.pbuf.copy_(torch.stack([self.embed(torch.tensor(k)) for k in ids]))
        self.pbuf.copy_(self.layers(self.pbuf, -1))
        if self.last:
            self.hidden[b][i].copy_(self.pbuf[-1])

    def head_input(self, b):
        return self.hidden[b] if self.last else self.head_in[b]

    def head_keys(self, b):
        return self.keys[b][0]

    def gathered_keys(self, b, s):
        return self.keys[b][s]

    def run_head_shard(self, b):
        for i in range(self.mb_size):
            target = int(self.sample(self.head_input(b)[i])[0])
            best = 0
            for v in range(self.v0, self.v1):
                key = ((V - abs(v - target)) << 32) | (0xFFFFFFFF - v)
                best = max(best, key)
            self.keys[b][0][i] = best

    def merge(self, b):
        for i in range(self.mb_size):
            k = int(self.keys[b][:, i].max())
            self.tokens[b][i] = 0xFFFFFFFF - (k & 0xFFFFFFFF)


def _vocab_worker(rank, world, port, n_mb, R, prompts, steps, result_dir, shares):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.model import vocab_shards
    from dial_cuda.pipeline import Pipeline, TorchChannel, head_links, init_distributed
    init_distributed("gloo", timeout_s=30)
    spans = vocab_shards(V, shares)
    rows = [v1 - v0 for v0, v1 in spans]
    c = FakeVocabCompute(rank, world, n_mb, R, spans[rank])
    hch = TorchChannel(world, links=head_links(world, rows))
    p = Pipeline(rank, world, c, TorchChannel(world), n_mb, head_channel=hch, head_rows=rows)
    p.prefill(prompts if rank == 0 else None, prompt_len=len(prompts[0]))
    firsts = [int(v) for t in c.tokens for v in t.reshape(-1)]
    p.steps(2)
    p.steps(steps - 2)
    p.finish()
    torch.save({"firsts": firsts, "after_finish": [int(v) for t in c.tokens for v in t.reshape(-1)]},
               os.path.join(result_dir, f"v{rank}.pt"))
    import torch.distributed as dist
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,shares", [(2, [1, 1]), (3, [1, 2, 1]), (4, [0, 1, 0, 3]),
                                          (4, [1, 1, 1, 0])])
def test_vocab_parallel_head_matches_single_process_chain(world, shares, tmp_path):
    """The head split over the stages by vocabulary rows (uneven shares, stages
    with none, the last stage with none): the tokens merged on stage 0 after
    prefill and after the decode steps equal the single-process chain's."""
    n_mb, R, steps = max(3, world), 2, 5
    prompts = [[(3 * s + 7 * i + 1) % V for i in range(4)] for s in range(n_mb * R)]
    mp.start_processes(_vocab_worker,
                       args=(world, _free_port(), n_mb, R, prompts, steps, str(tmp_path), shares),
                       nprocs=world, join=True, start_method="spawn")
    ref = reference(world, n_mb * R, prompts, steps)
    r0 = torch.load(tmp_path / "v0.pt")
    assert r0["firsts"] == [seq[0] for seq in ref]
    assert r0["after_finish"] == [seq[-1] for seq in ref]


def test_vocab_shards_and_head_links():
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.model import vocab_shards
    from dial_cuda.pipeline import head_links
    spans = vocab_shards(151936, [1] * 8)
    assert spans[0][0] == 0 and spans[-1][1] == 151936
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all((v1 - v0) % 16 == 0 for v0, v1 in spans[:-1])
    assert vocab_shards(100, [0, 1, 0]) == [(0, 0), (0, 100), (100, 100)]
    assert head_links(4, [1, 1, 1, 1]) == [(3, 0), (3, 1), (3, 2), (1, 0), (2, 0)]
    assert head_links(4, [0, 1, 0, 3]) == [(3, 1), (1, 0), (3, 0)]
    assert head_links(3, [5, 5, 0]) == [(2, 0), (2, 1), (1, 0)]
