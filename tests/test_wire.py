"""The reference's TCP framing and message kinds (spm/proto/message.rs) and the
pipeline over TCP links: framing limits, every message kind through the body
codec, the transfer limiter's environment and pacing, and 2- and 3-stage
pipelines over TcpChannel checked against the single-process chain."""
import os
import socket
import struct
import sys

import pytest

import torch
import torch.multiprocessing as mp

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "dial-8b-orin_b200"))
from dial_cuda import wire as W  # noqa: E402

from test_pipeline_cpu import FakeCompute, _free_port, reference  # noqa: E402


def _pair():
    a, b = socket.socketpair()
    return a, b


def _roundtrip(m):
    a, b = _pair()
    try:
        n = W.write_message(a, m, limiter=None)
        size, got = W.read_message(b)
        assert n == 8 + size
        return got
    finally:
        a.close()
        b.close()


def test_header_is_big_endian_magic_and_length():
    a, b = _pair()
    W.write_message(a, W.Message.hello(), limiter=None)
    head = b.recv(8)
    assert struct.unpack(">II", head) == (0x104F4C7, 1)  # Hello: one variant byte
    assert head[:4] == bytes([0x01, 0x04, 0xF4, 0xC7])
    a.close()
    b.close()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64,
                                   torch.uint8, torch.int64])
def test_tensor_message_round_trip(dtype):
    x = (torch.arange(24, dtype=torch.float64) * 0.37 - 3.0).to(dtype).view(2, 3, 4)
    got = _roundtrip(W.Message.from_tensor(x, compute_us=1234))
    assert got.kind == "Tensor" and got.compute_us == 1234
    assert got.x.shape == (2, 3, 4)
    y = got.x.to_tensor()
    assert y.dtype == dtype and torch.equal(y.view(torch.uint8), x.view(torch.uint8))


def test_token_ids_travel_as_u32():
    ids = torch.tensor([0, 7, 151935], dtype=torch.int32)
    got = _roundtrip(W.Message.from_tensor(ids))
    assert got.x.dtype == "U32"
    out = torch.zeros(3, dtype=torch.int32)
    got.x.to_tensor(out=out)
    assert out.tolist() == [0, 7, 151935]


def test_every_message_kind_round_trips():
    x = W.RawTensor.from_tensor(torch.ones(1, 4, dtype=torch.float16))
    s = W.SamplingRequest(seed=299792458, sample_index=3, temperature=0.7, top_k=40, top_p=None,
                          repeat_penalty=1.25, repeat_context=[1, 2, 3])  # f32 field: exact value
    msgs = [
        W.Message.hello(),
        W.Message("WorkerInfo", info=W.WorkerInfo(version="0.3|w8a16|gguf", dtype="f16", os="linux",
                                                  arch="x86_64", device="cuda", device_idx=1,
                                                  latency=2 ** 70 + 5, cpu_usage_percent=12.5,
                                                  system_model="B200")),
        W.Message("SingleOp", layer_name="model.layers.3", x=x, index_pos=17, block_idx=3, sampling=s),
        W.Message("Batch", x=x, batch=[("model.layers.0", 5, 0), ("model.layers.1", 5, 1)]),
        W.Message("CompactBatch", x=x, batch=W.CompactBatch("model.layers.4", 9, 4, 12), sampling=s),
        W.Message("CompactRangeBatch", x=x, batch=W.CompactRangeBatch(9, 18, 18)),
        W.Message("Tensor", x=x, compute_us=77),
    ]
    for m in msgs:
        assert _roundtrip(m) == m
    info = msgs[1].info
    assert info.supports("gguf") and info.supports("w8a16") and not info.supports("0.3")


def test_reader_rejects_bad_magic_and_oversized_length():
    for head, what in ((struct.pack(">II", 0xDEADBEEF, 1), "invalid magic value"),
                       (struct.pack(">II", W.PROTO_MAGIC, W.MESSAGE_MAX_SIZE + 1), "MESSAGE_MAX_SIZE")):
        a, b = _pair()
        a.sendall(head)
        with pytest.raises(W.WireError, match=what):
            W.read_message(b)
        a.close()
        b.close()


def test_writer_refuses_an_oversized_body():
    with pytest.raises(W.WireError, match="MESSAGE_MAX_SIZE"):
        W.frame_header(W.MESSAGE_MAX_SIZE + 1)
    assert W.frame_header(W.MESSAGE_MAX_SIZE)[4:] == struct.pack(">I", W.MESSAGE_MAX_SIZE)


def test_truncated_and_malformed_bodies_are_errors():
    body = W.encode_body(W.Message.from_tensor(torch.ones(3)))
    with pytest.raises(W.WireError, match="ends early"):
        W.decode_body(body[:-3])
    with pytest.raises(W.WireError, match="after the message"):
        W.decode_body(body + b"\x00")
    with pytest.raises(W.WireError, match="unknown message variant"):
        W.decode_body(b"\x07")
    a, b = _pair()
    a.sendall(struct.pack(">II", W.PROTO_MAGIC, 100) + body[:10])
    a.close()
    with pytest.raises(W.WireError, match="connection closed"):
        W.read_message(b)
    b.close()


def test_unsupported_dtype_and_mismatched_buffer():
    with pytest.raises(W.WireError, match="unsupported tensor dtype"):
        W.RawTensor.from_tensor(torch.ones(2, dtype=torch.complex64))
    r = W.RawTensor.from_tensor(torch.ones(2, 4, dtype=torch.float16))
    with pytest.raises(W.WireError, match="shape"):
        r.to_tensor(out=torch.zeros(4, 2, dtype=torch.float16))
    with pytest.raises(W.WireError, match="dtype"):
        r.to_tensor(out=torch.zeros(2, 4, dtype=torch.bfloat16))


def test_limiter_environment():
    f = W.TransferLimiter.from_env
    assert f({}) is None
    lim = f({"SPM_TRANSFER_LIMIT_MBPS": "8"})
    assert lim.bytes_per_sec == 1_000_000.0 and lim.chunk_bytes == 65536  # 100 KB clamped
    lim = f({"SPM_TRANSFER_LIMIT_KBPS": "80"})
    assert lim.bytes_per_sec == 10_000.0 and lim.chunk_bytes == 1024  # 1 KB floor
    lim = f({"SPM_TRANSFER_LIMIT_BYTES_PER_SEC": "200000", "SPM_TRANSFER_LIMIT_CHUNK_BYTES": "300"})
    assert lim.bytes_per_sec == 200_000.0 and lim.chunk_bytes == 300
    # MBPS wins over the others; a bad number falls through; non-positive disables
    assert f({"SPM_TRANSFER_LIMIT_MBPS": "1", "SPM_TRANSFER_LIMIT_KBPS": "5"}).bytes_per_sec == 125_000.0
    assert f({"SPM_TRANSFER_LIMIT_MBPS": "x", "SPM_TRANSFER_LIMIT_KBPS": "8"}).bytes_per_sec == 1000.0
    assert f({"SPM_TRANSFER_LIMIT_MBPS": "0"}) is None
    assert f({"SPM_TRANSFER_LIMIT_MBPS": "-3"}) is None
    assert f({"SPM_TRANSFER_LIMIT_BYTES_PER_SEC": "1000", "SPM_TRANSFER_LIMIT_CHUNK_BYTES": "0.5"}).chunk_bytes == 1024


def test_limiter_paces_chunks():
    now = [100.0]
    slept = []

    def sleep(d):
        slept.append(round(d, 9))
        now[0] += d
    lim = W.TransferLimiter(1000.0, 250, clock=lambda: now[0], sleep=sleep)

    class Sink:
        def __init__(self):
            self.writes = []

        def sendall(self, b):
            self.writes.append(len(b))
    s = Sink()
    W._write_all(s, b"x" * 1000, lim)
    assert s.writes == [250, 250, 250, 250]
    assert slept == [0.25, 0.25, 0.25]  # the first chunk goes at once, then one chunk per 0.25 s
    now[0] += 5.0  # idle time is not banked: the next chunk waits for nothing
    W._write_all(s, b"x" * 100, lim)
    assert slept == [0.25, 0.25, 0.25]


def _tcp_worker(rank, world, ports, n_mb, prompts, steps, result_dir):
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from dial_cuda.pipeline import Pipeline
    from dial_cuda.wire import TcpChannel
    ch = TcpChannel(rank, world, [("127.0.0.1", p) for p in ports], timeout_s=30.0, limiter=None)
    c = FakeCompute(rank, world, n_mb)
    p = Pipeline(rank, world, c, ch, n_mb)
    p.prefill(prompts if rank == 0 else None, prompt_len=len(prompts[0]))
    firsts = [int(v) for t in c.tokens for v in t.reshape(-1)]
    p.steps(2)
    p.steps(steps - 2)
    last = [int(v) for t in c.tokens for v in t.reshape(-1)]
    p.finish()
    ch.close()
    torch.save({"firsts": firsts, "last": last,
                "after_finish": [int(v) for t in c.tokens for v in t.reshape(-1)]},
               os.path.join(result_dir, f"r{rank}.pt"))


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_over_tcp_matches_single_process_chain(world, tmp_path):
    n_mb, steps = 3, 5
    prompts = [[(7 * b + 3 * i) % 97 for i in range(4)] for b in range(n_mb)]
    ports = [_free_port() for _ in range(world)]
    mp.start_processes(_tcp_worker, args=(world, ports, n_mb, prompts, steps, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    ref = reference(world, n_mb, prompts, steps)
    r0 = torch.load(tmp_path / "r0.pt")
    rl = torch.load(tmp_path / f"r{world - 1}.pt")
    assert r0["firsts"] == [seq[0] for seq in ref]
    assert rl["last"] == [seq[-1] for seq in ref]
    assert r0["after_finish"] == [seq[-1] for seq in ref]


def _tcp_vocab_worker(rank, world, ports, head_ports, n_mb, R, prompts, steps, result_dir, shares):
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "dial-8b-orin_b200"))
    from test_pipeline_cpu import FakeVocabCompute, V
    from dial_cuda.model import vocab_shards
    from dial_cuda.pipeline import Pipeline, head_links
    from dial_cuda.wire import TcpChannel
    spans = vocab_shards(V, shares)
    rows = [v1 - v0 for v0, v1 in spans]
    ch = TcpChannel(rank, world, [("127.0.0.1", p) for p in ports], timeout_s=30.0, limiter=None)
    hch = TcpChannel(rank, world, [("127.0.0.1", p) for p in head_ports],
                     links=head_links(world, rows), timeout_s=30.0, limiter=None)
    c = FakeVocabCompute(rank, world, n_mb, R, spans[rank])
    p = Pipeline(rank, world, c, ch, n_mb, head_channel=hch, head_rows=rows)
    p.prefill(prompts if rank == 0 else None, prompt_len=len(prompts[0]))
    firsts = [int(v) for t in c.tokens for v in t.reshape(-1)]
    p.steps(steps)
    p.finish()
    ch.close()
    hch.close()
    torch.save({"firsts": firsts, "after_finish": [int(v) for t in c.tokens for v in t.reshape(-1)]},
               os.path.join(result_dir, f"v{rank}.pt"))


@pytest.mark.parametrize("world,shares", [(2, [1, 1]), (3, [1, 2, 0])])
def test_vocab_parallel_head_over_tcp(world, shares, tmp_path):
    """The vocabulary-parallel head's exchange (hidden states to the shard
    stages, greedy keys to stage 0) over a second set of TCP links."""
    n_mb, R, steps = max(3, world), 2, 4
    V = 97
    prompts = [[(3 * s + 7 * i + 1) % V for i in range(4)] for s in range(n_mb * R)]
    ports = [_free_port() for _ in range(world)]
    head_ports = [_free_port() for _ in range(world)]
    mp.start_processes(_tcp_vocab_worker,
                       args=(world, ports, head_ports, n_mb, R, prompts, steps, str(tmp_path), shares),
                       nprocs=world, join=True, start_method="spawn")
    ref = reference(world, n_mb * R, prompts, steps)
    r0 = torch.load(tmp_path / "v0.pt")
    assert r0["firsts"] == [seq[0] for seq in ref]
    assert r0["after_finish"] == [seq[-1] for seq in ref]


def test_missing_tcp_peer_times_out():
    port = _free_port()  # nothing listens there
    with pytest.raises(TimeoutError, match="no listener"):
        W.TcpChannel(0, 2, [("127.0.0.1", _free_port()), ("127.0.0.1", port)], timeout_s=0.5, limiter=None)


@pytest.mark.gpu
def test_tcp_channel_carries_device_buffers():
    """Two stages in two threads of one process on one GPU: a bf16 hidden state
    forward and int32 token ids back, device -> pinned host -> TCP -> device,
    bit-exact and in order over repeated transfers."""
    import threading
    addrs = [("127.0.0.1", _free_port()), ("127.0.0.1", _free_port())]
    chans = [None, None]

    def make(r):
        chans[r] = W.TcpChannel(r, 2, addrs, timeout_s=20.0, limiter=None)
    th = [threading.Thread(target=make, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    c0, c1 = chans
    g = torch.Generator(device="cuda").manual_seed(299792458)
    try:
        for step in range(3):
            h = torch.randn(4, 4096, device="cuda", generator=g).to(torch.bfloat16)
            ids = torch.randint(0, 151936, (4,), device="cuda", generator=g, dtype=torch.int32)
            got_h = torch.empty_like(h)
            got_ids = torch.zeros_like(ids)
            done = [c0.isend(h, 1), c1.irecv(got_h, 0), c1.isend(ids, 0), c0.irecv(got_ids, 1)]
            for d in done:
                d.wait()
            torch.cuda.synchronize()
            assert torch.equal(got_h.view(torch.int16), h.view(torch.int16)), step
            assert torch.equal(got_ids, ids), step
    finally:
        c0.close()
        c1.close()


# ---------------------------------------------------------------- master/worker exchange
def _fake_run(x, first, n, index_pos):
    y = x.clone().double()
    for blk in range(first, first + n):
        y = y * 0.75 + 0.125 * (blk + 1) + 0.01 * index_pos
    return y.to(x.dtype)


def _serve_once(worker):
    """A listener on a free port; the worker serves its first connection in a thread."""
    import threading
    srv = socket.create_server(("127.0.0.1", 0))
    box = {}

    def go():
        s, _ = srv.accept()
        try:
            box["served"] = worker.serve(s, limiter=None)
        except Exception as e:  # noqa: BLE001 -- checked by the test
            box["error"] = e
        finally:
            s.close()
            srv.close()
    th = threading.Thread(target=go, daemon=True)
    th.start()
    return srv.getsockname(), th, box


NAMES = {b: f"model.layers.{b}" for b in range(8, 14)}


def test_compact_batch_names_follow_the_first_name():
    assert W.expand_compact_batch("model.layers.7", 5, 7, 3) == [
        ("model.layers.7", 5, 7), ("model.layers.8", 5, 8), ("model.layers.9", 5, 9)]
    with pytest.raises(W.WireError, match="numeric suffix"):
        W.expand_compact_batch("model.layers.x", 0, 0, 1)
    m = W.Message("CompactRangeBatch", batch=W.CompactRangeBatch(3, 12, 3))
    with pytest.raises(W.WireError, match="missing local block index 14"):
        W.request_ops(m, NAMES)


@pytest.mark.parametrize("caps,kind", [(W.WORKER_CAPABILITIES, "CompactRangeBatch"),
                                       (("compact_batch_v1",), "CompactBatch"), ((), "Batch")])
def test_master_worker_exchange(caps, kind):
    """The master's request kind follows the worker's advertised capabilities;
    every kind runs the same blocks and returns the same hidden state."""
    info = W.WorkerInfo(version="dial-b200|" + "|".join(caps))
    addr, th, box = _serve_once(W.StageWorker(_fake_run, NAMES, info))
    cl = W.RemoteStage(addr, timeout_s=10.0, limiter=None)
    assert cl.info.version == info.version
    x = torch.randn(1, 5, 64).to(torch.bfloat16)
    for index_pos in (0, 5):  # a prompt, then the next position
        batch = [(NAMES[b], index_pos, b) for b in range(9, 13)]
        y = cl.forward_batch(x, batch)
        assert cl.last_kind == kind
        assert torch.equal(y.view(torch.int16), _fake_run(x, 9, 4, index_pos).view(torch.int16))
    out = torch.empty_like(x)
    cl.forward_batch(x, [(NAMES[8], 2, 8)], out=out)  # one block
    assert torch.equal(out.view(torch.int16), _fake_run(x, 8, 1, 2).view(torch.int16))
    cl.close()
    th.join(timeout=10)
    assert box.get("served") == 3, box


def test_worker_rejects_foreign_and_scattered_blocks():
    for batch, what in (([("model.layers.20", 0, 20)], "missing local block index 20"),
                        ([("model.layers.8", 0, 8), ("model.layers.10", 0, 10)], "contiguous")):
        addr, th, box = _serve_once(W.StageWorker(_fake_run, NAMES))
        cl = W.RemoteStage(addr, timeout_s=10.0, limiter=None)
        with pytest.raises(W.WireError):
            cl.forward_batch(torch.ones(1, 1, 8), batch)  # the worker drops the connection
        cl.close()
        th.join(timeout=10)
        assert what in str(box.get("error")), box


def test_worker_wants_hello_first():
    addr, th, box = _serve_once(W.StageWorker(_fake_run, NAMES))
    s = socket.create_connection(addr)
    W.write_message(s, W.Message.from_tensor(torch.ones(2)), limiter=None)
    th.join(timeout=10)
    s.close()
    assert "instead of hello" in str(box.get("error")), box



def test_send_wait_is_bounded():
    """A frame the writer thread never finishes (a peer that stops reading)
    ends the sender's wait with a timeout instead of blocking it."""
    import queue
    d = W._Sent(queue.Queue(), 0.2, (0, 1))
    with pytest.raises(TimeoutError, match="not written within"):
        d.wait()
    q = queue.Queue()
    q.put(None)
    done = W._Sent(q, 0.2, (0, 1))
    done.wait()
    done.wait()  # a finished send may be waited on again
