"""The reference's TCP protocol for stages on hosts that NVLink does not join.

The reference frames every master/worker message as

    [magic u32 big-endian = 0x104F4C7][length u32 big-endian][body]

(`dial-core/src/spm/proto/message.rs:366-408`, constants in
`dial-core/src/spm/proto/mod.rs:4-7`): a reader rejects another magic and a
length above 512 MiB, a writer refuses to send a larger body, and the header
and the body are written as two writes, optionally paced by a token-bucket
limiter read from the environment (`message.rs:16-99`).  The message kinds
and their fields are those of `Message`, `RawTensor`, `RawDType`,
`CompactBatch`, `CompactRangeBatch` and `SamplingRequest` (`message.rs:101-235`).

The body: the reference serialises `Message` with the `bitcode` crate
(0.6.6, `Cargo.lock:375-378`, not vendored; no golden bytes exist in the
reference's tests), whose packed layout cannot be restated and checked here.
This module writes the same fields in a fixed little-endian layout instead
(`encode_body` / `decode_body`): one variant byte in the reference's enum
order, u64 for `usize`/`u64`, IEEE floats, `u64` length + bytes for strings
and vectors, one presence byte for `Option`.  The framing, limits, pacing and
message semantics are the reference's; a Rust host that keeps its own
`message.rs` talks to this module only once both ends use one body codec.

`TcpChannel` carries the pipeline's hand-off (`dial_cuda.pipeline.Pipeline`)
over these frames: every transfer is one `Message::Tensor` whose `RawTensor`
holds the hidden state (or the token ids) in the sender's dtype and shape,
copied device -> pinned host -> socket on the sender and back on the receiver,
as the reference's `RawTensor::from_tensor` / `to_tensor` do at every stage
boundary (`message.rs:147-165`, `worker.rs:700-760`)."""
from __future__ import annotations

import os
import queue
import socket
import struct
import threading
import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

PROTO_MAGIC = 0x104F4C7           # spm/proto/mod.rs:4
MESSAGE_MAX_SIZE = 512 * 1024 * 1024  # spm/proto/mod.rs:7

# RawDType in the reference's order (message.rs:101-110)
RAW_DTYPES = ("F16", "BF16", "F32", "F64", "U8", "U32", "I64")
# Message variants in the reference's order (message.rs:235-272)
VARIANTS = ("Hello", "WorkerInfo", "SingleOp", "Batch", "CompactBatch", "CompactRangeBatch", "Tensor")


class WireError(RuntimeError):
    """A malformed, oversized or unexpected message."""


class ConnectionClosed(WireError):
    """The peer closed the connection between two messages."""


def _torch():
    import torch  # noqa: PLC0415
    return torch


def _torch_dtypes():
    torch = _torch()
    return {"F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
            "U8": torch.uint8, "U32": torch.uint32, "I64": torch.int64}


def raw_dtype_of(dtype) -> str:
    """RawDType::from_dtype (message.rs:113-125): the dtypes the protocol carries."""
    for name, dt in _torch_dtypes().items():
        if dt == dtype:
            return name
    if dtype == _torch().int32:  # token ids travel as u32, as the reference's token tensors are
        return "U32"
    raise WireError(f"unsupported tensor dtype in SPM protocol: {dtype}")


# ---------------------------------------------------------------- message types
@dataclass
class RawTensor:
    """A tensor's bytes, dtype and shape (message.rs:137-165)."""
    data: bytes
    dtype: str
    shape: Tuple[int, ...]

    @staticmethod
    def from_tensor(x, pinned=None) -> "RawTensor":
        """Copies x (any device) to host bytes; `pinned` (a uint8 host tensor of
        at least x's bytes, page-locked) stages a device copy."""
        torch = _torch()
        dt = raw_dtype_of(x.dtype)
        x = x.contiguous()
        nbytes = x.numel() * x.element_size()
        if x.is_cuda:
            if pinned is not None and pinned.numel() >= nbytes:
                host = pinned[:nbytes]
                host.copy_(x.view(-1).view(torch.uint8))  # synchronises with x's stream
            else:
                host = x.view(-1).view(torch.uint8).cpu()
        else:
            host = x.view(-1).view(torch.uint8)
        return RawTensor(host.numpy().tobytes(), dt, tuple(int(s) for s in x.shape))

    def to_tensor(self, device=None, out=None):
        """A tensor of this dtype and shape; with `out`, copies into it (its
        dtype may be int32 for U32 ids) and checks shape and size."""
        torch = _torch()
        n = 1
        for s in self.shape:
            n *= s
        host = torch.frombuffer(bytearray(self.data), dtype=torch.uint8) if self.data else \
            torch.empty(0, dtype=torch.uint8)
        if out is not None:
            if tuple(out.shape) != tuple(self.shape):
                raise WireError(f"tensor shape {self.shape} does not match the receive buffer {tuple(out.shape)}")
            if raw_dtype_of(out.dtype) != self.dtype:
                raise WireError(f"tensor dtype {self.dtype} does not match the receive buffer {out.dtype}")
            if host.numel() != out.numel() * out.element_size():
                raise WireError("tensor data size does not match its shape")
            out.view(-1).view(torch.uint8).copy_(host, non_blocking=out.is_cuda)
            return out
        dt = _torch_dtypes()[self.dtype]
        elt = torch.empty(0, dtype=dt).element_size()
        if host.numel() != n * elt:
            raise WireError("tensor data size does not match its shape")
        t = host.view(dt).view(self.shape) if n else torch.empty(self.shape, dtype=dt)
        return t.to(device) if device is not None else t


@dataclass
class SamplingRequest:
    """message.rs:181-190."""
    seed: int = 0
    sample_index: int = 0
    temperature: float = 0.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None
    repeat_penalty: float = 1.0
    repeat_context: List[int] = field(default_factory=list)


@dataclass
class CompactBatch:
    first_layer_name: str
    index_pos: int
    first_block_idx: int
    num_layers: int


@dataclass
class CompactRangeBatch:
    index_pos: int
    first_block_idx: int
    num_layers: int


@dataclass
class WorkerInfo:
    """message.rs:192-217 (diagnostics a worker sends after Hello)."""
    version: str = ""
    dtype: str = ""
    os: str = ""
    arch: str = ""
    device: str = ""
    device_idx: int = 0
    latency: int = 0
    cpu_usage_percent: Optional[float] = None
    memory_usage_percent: Optional[float] = None
    npu_usage_percent: Optional[float] = None
    temperature_c: Optional[float] = None
    system_model: Optional[str] = None

    def supports(self, capability: str) -> bool:
        """message.rs:219-227: capabilities follow the version, '|'-separated."""
        return capability in self.version.split("|")[1:]


@dataclass
class Message:
    """One of VARIANTS with its fields (message.rs:235-272):
    Hello; WorkerInfo(info); SingleOp(layer_name, x, index_pos, block_idx,
    sampling); Batch(x, batch [(name, index_pos, block_idx)], sampling);
    CompactBatch(x, batch, sampling); CompactRangeBatch(x, batch, sampling);
    Tensor(x, compute_us)."""
    kind: str
    x: Optional[RawTensor] = None
    info: Optional[WorkerInfo] = None
    layer_name: str = ""
    index_pos: int = 0
    block_idx: int = 0
    batch: object = None
    sampling: Optional[SamplingRequest] = None
    compute_us: int = 0

    @staticmethod
    def hello() -> "Message":
        return Message("Hello")

    @staticmethod
    def from_tensor(x, compute_us: int = 0, pinned=None) -> "Message":
        """Message::from_tensor_with_compute (message.rs:284-296)."""
        return Message("Tensor", x=RawTensor.from_tensor(x, pinned), compute_us=compute_us)


# ---------------------------------------------------------------- body codec
class _W:
    def __init__(self):
        self.parts = []

    def u8(self, v):
        self.parts.append(struct.pack("<B", v))

    def u64(self, v):
        if v < 0:
            raise WireError(f"negative value {v} for an unsigned field")
        self.parts.append(struct.pack("<Q", v))

    def f32(self, v):
        self.parts.append(struct.pack("<f", v))

    def f64(self, v):
        self.parts.append(struct.pack("<d", v))

    def bytes_(self, b):
        self.u64(len(b))
        self.parts.append(bytes(b))

    def str_(self, s):
        self.bytes_(s.encode("utf-8"))

    def opt(self, v, fn):
        self.u8(0 if v is None else 1)
        if v is not None:
            fn(v)

    def tensor(self, t: RawTensor):
        self.bytes_(t.data)
        if t.dtype not in RAW_DTYPES:
            raise WireError(f"unsupported tensor dtype in SPM protocol: {t.dtype}")
        self.u8(RAW_DTYPES.index(t.dtype))
        self.u64(len(t.shape))
        for s in t.shape:
            self.u64(s)

    def sampling(self, s: Optional[SamplingRequest]):
        def one(v):
            self.u64(v.seed)
            self.u64(v.sample_index)
            self.f64(v.temperature)
            self.opt(v.top_k, self.u64)
            self.opt(v.top_p, self.f64)
            self.f32(v.repeat_penalty)
            self.u64(len(v.repeat_context))
            for c in v.repeat_context:
                self.parts.append(struct.pack("<I", c))
        self.opt(s, one)


class _R:
    def __init__(self, b: bytes):
        self.b, self.i = memoryview(b), 0

    def take(self, n):
        if self.i + n > len(self.b):
            raise WireError("message body ends early")
        v = self.b[self.i:self.i + n]
        self.i += n
        return v

    def u8(self):
        return self.take(1)[0]

    def u64(self):
        return struct.unpack("<Q", self.take(8))[0]

    def f32(self):
        return struct.unpack("<f", self.take(4))[0]

    def f64(self):
        return struct.unpack("<d", self.take(8))[0]

    def bytes_(self):
        return bytes(self.take(self.u64()))

    def str_(self):
        return self.bytes_().decode("utf-8")

    def opt(self, fn):
        flag = self.u8()
        if flag > 1:
            raise WireError(f"bad option flag {flag}")
        return fn() if flag else None

    def tensor(self) -> RawTensor:
        data = self.bytes_()
        d = self.u8()
        if d >= len(RAW_DTYPES):
            raise WireError(f"unknown tensor dtype code {d}")
        shape = tuple(self.u64() for _ in range(self.u64()))
        return RawTensor(data, RAW_DTYPES[d], shape)

    def sampling(self) -> Optional[SamplingRequest]:
        def one():
            s = SamplingRequest(self.u64(), self.u64(), self.f64())
            s.top_k = self.opt(self.u64)
            s.top_p = self.opt(self.f64)
            s.repeat_penalty = self.f32()
            s.repeat_context = [struct.unpack("<I", self.take(4))[0] for _ in range(self.u64())]
            return s
        return self.opt(one)


def encode_body(m: Message) -> bytes:
    if m.kind not in VARIANTS:
        raise WireError(f"unknown message kind {m.kind!r}")
    w = _W()
    w.u8(VARIANTS.index(m.kind))
    if m.kind == "WorkerInfo":
        i = m.info or WorkerInfo()
        for s in (i.version, i.dtype, i.os, i.arch, i.device):
            w.str_(s)
        w.u64(i.device_idx)
        w.bytes_(int(i.latency).to_bytes(16, "little"))  # u128
        for v in (i.cpu_usage_percent, i.memory_usage_percent, i.npu_usage_percent, i.temperature_c):
            w.opt(v, w.f32)
        w.opt(i.system_model, w.str_)
    elif m.kind == "SingleOp":
        w.str_(m.layer_name)
        w.tensor(m.x)
        w.u64(m.index_pos)
        w.u64(m.block_idx)
        w.sampling(m.sampling)
    elif m.kind == "Batch":
        w.tensor(m.x)
        w.u64(len(m.batch))
        for name, ip, bi in m.batch:
            w.str_(name)
            w.u64(ip)
            w.u64(bi)
        w.sampling(m.sampling)
    elif m.kind == "CompactBatch":
        w.tensor(m.x)
        b = m.batch
        w.str_(b.first_layer_name)
        w.u64(b.index_pos)
        w.u64(b.first_block_idx)
        w.u64(b.num_layers)
        w.sampling(m.sampling)
    elif m.kind == "CompactRangeBatch":
        w.tensor(m.x)
        b = m.batch
        w.u64(b.index_pos)
        w.u64(b.first_block_idx)
        w.u64(b.num_layers)
        w.sampling(m.sampling)
    elif m.kind == "Tensor":
        w.tensor(m.x)
        w.u64(m.compute_us)
    return b"".join(w.parts)


def decode_body(raw: bytes) -> Message:
    r = _R(raw)
    v = r.u8()
    if v >= len(VARIANTS):
        raise WireError(f"unknown message variant {v}")
    kind = VARIANTS[v]
    m = Message(kind)
    if kind == "WorkerInfo":
        i = WorkerInfo(*(r.str_() for _ in range(5)))
        i.device_idx = r.u64()
        i.latency = int.from_bytes(r.bytes_(), "little")
        i.cpu_usage_percent, i.memory_usage_percent, i.npu_usage_percent, i.temperature_c = (
            r.opt(r.f32) for _ in range(4))
        i.system_model = r.opt(r.str_)
        m.info = i
    elif kind == "SingleOp":
        m.layer_name = r.str_()
        m.x = r.tensor()
        m.index_pos, m.block_idx = r.u64(), r.u64()
        m.sampling = r.sampling()
    elif kind == "Batch":
        m.x = r.tensor()
        m.batch = [(r.str_(), r.u64(), r.u64()) for _ in range(r.u64())]
        m.sampling = r.sampling()
    elif kind == "CompactBatch":
        m.x = r.tensor()
        m.batch = CompactBatch(r.str_(), r.u64(), r.u64(), r.u64())
        m.sampling = r.sampling()
    elif kind == "CompactRangeBatch":
        m.x = r.tensor()
        m.batch = CompactRangeBatch(r.u64(), r.u64(), r.u64())
        m.sampling = r.sampling()
    elif kind == "Tensor":
        m.x = r.tensor()
        m.compute_us = r.u64()
    if r.i != len(r.b):
        raise WireError(f"{len(r.b) - r.i} bytes after the message")
    return m


# ---------------------------------------------------------------- pacing
class TransferLimiter:
    """message.rs:16-73: SPM_TRANSFER_LIMIT_MBPS (megabit/s), else _KBPS
    (kilobit/s), else _BYTES_PER_SEC; SPM_TRANSFER_LIMIT_CHUNK_BYTES, else a
    tenth of a second's bytes clamped to [1024, 65536].  Each chunk waits for
    its slot: the later of now and the end of the previous chunk's transfer."""

    def __init__(self, bytes_per_sec: float, chunk_bytes: int, clock=time.monotonic, sleep=time.sleep):
        self.bytes_per_sec, self.chunk_bytes = bytes_per_sec, chunk_bytes
        self.clock, self.sleep = clock, sleep
        self.next_write_at = clock()
        self.lock = threading.Lock()

    @staticmethod
    def from_env(env=None, **kw) -> Optional["TransferLimiter"]:
        env = os.environ if env is None else env

        def num(name):
            try:
                return float(env[name].strip())
            except (KeyError, ValueError):
                return None
        if (v := num("SPM_TRANSFER_LIMIT_MBPS")) is not None:
            bps = v * 1_000_000.0 / 8.0
        elif (v := num("SPM_TRANSFER_LIMIT_KBPS")) is not None:
            bps = v * 1_000.0 / 8.0
        elif (v := num("SPM_TRANSFER_LIMIT_BYTES_PER_SEC")) is not None:
            bps = v
        else:
            return None
        if not (bps > 0.0 and bps != float("inf")):
            return None
        c = num("SPM_TRANSFER_LIMIT_CHUNK_BYTES")
        if c is not None and c >= 1.0 and c != float("inf"):
            chunk = int(c)
        else:
            chunk = min(max(int(round(bps / 10.0)), 1024), 64 * 1024)
        return TransferLimiter(bps, chunk, **kw)

    def wait_for_slot(self, nbytes: int) -> None:
        now = self.clock()
        with self.lock:
            start = max(self.next_write_at, now)
            self.next_write_at = start + nbytes / self.bytes_per_sec
        if start > now:
            self.sleep(start - now)


_LIMITER_UNSET = object()
_limiter = _LIMITER_UNSET


def transfer_limiter() -> Optional[TransferLimiter]:
    """The process's limiter, read from the environment once (message.rs:75-78)."""
    global _limiter
    if _limiter is _LIMITER_UNSET:
        _limiter = TransferLimiter.from_env()
    return _limiter


def _write_all(sock, data, limiter) -> None:
    if limiter is None:
        sock.sendall(data)
        return
    mv = memoryview(data)
    for i in range(0, len(mv), limiter.chunk_bytes):
        chunk = mv[i:i + limiter.chunk_bytes]
        limiter.wait_for_slot(len(chunk))
        sock.sendall(chunk)


# ---------------------------------------------------------------- framing
def frame_header(body_len: int) -> bytes:
    if body_len > MESSAGE_MAX_SIZE:
        raise WireError(f"request size {body_len} > MESSAGE_MAX_SIZE")
    return struct.pack(">II", PROTO_MAGIC, body_len)


def write_message(sock, m: Message, limiter=_LIMITER_UNSET) -> int:
    """Message::to_writer (message.rs:390-408): header then body; returns the
    bytes written."""
    body = encode_body(m)
    header = frame_header(len(body))
    lim = transfer_limiter() if limiter is _LIMITER_UNSET else limiter
    _write_all(sock, header, lim)
    _write_all(sock, body, lim)
    return 8 + len(body)


def _read_exact(sock, n: int, at_boundary: bool = False) -> bytes:
    buf = bytearray(n)
    mv, got = memoryview(buf), 0
    while got < n:
        k = sock.recv_into(mv[got:], n - got)
        if k == 0:
            if at_boundary and got == 0:
                raise ConnectionClosed("connection closed")
            raise WireError("connection closed inside a message")
        got += k
    return bytes(buf)


def read_message(sock) -> Tuple[int, Message]:
    """Message::from_reader (message.rs:366-388): (body bytes, message)."""
    magic, size = struct.unpack(">II", _read_exact(sock, 8, at_boundary=True))
    if magic != PROTO_MAGIC:
        raise WireError(f"invalid magic value: {magic}")
    if size > MESSAGE_MAX_SIZE:
        raise WireError(f"request size {size} > MESSAGE_MAX_SIZE")
    body = _read_exact(sock, size)
    return len(body), decode_body(body)


# ---------------------------------------------------------------- pipeline links over TCP
class _Sent:
    def __init__(self, fut, timeout_s, link):
        self.fut, self.timeout_s, self.link = fut, timeout_s, link

    def wait(self):
        try:
            err = self.fut.get(timeout=self.timeout_s)
        except queue.Empty:
            raise TimeoutError(f"link {self.link}: frame not written within {self.timeout_s} s") from None
        self.fut.put(err)  # wait() may be called again
        if err is not None:
            raise err


class _Received:
    def __init__(self, ch, link, t):
        self.ch, self.link, self.t, self.done = ch, link, t, False

    def wait(self):
        if self.done:
            return
        m = self.ch._next(self.link)
        if m.kind != "Tensor":
            raise WireError(f"expected a Tensor message on link {self.ch.links[self.link]}, got {m.kind}")
        m.x.to_tensor(out=self.t)
        self.done = True


class TcpChannel:
    """The pipeline's links (dial_cuda.pipeline.pipeline_links, or `links`)
    over TCP, for stages on different hosts.  Rank r listens on
    addrs[r] = (host, port); a link's sender connects to its receiver.  A send
    is framed and written by the link's writer thread (the caller's buffer is
    copied to host bytes first, on the caller's thread, so it can be reused at
    once); a receive takes the link's next message, read by its reader thread,
    and copies it into the buffer on the current stream.  Transfers on one
    link stay in order.  Every wait is bounded by timeout_s."""

    def __init__(self, rank: int, world: int, addrs: Sequence[Tuple[str, int]],
                 links: Optional[List[tuple]] = None, timeout_s: float = 60.0, limiter=_LIMITER_UNSET):
        from .pipeline import pipeline_links  # noqa: PLC0415
        self.rank, self.P, self.timeout_s = rank, world, timeout_s
        self.links = list(links) if links is not None else pipeline_links(world)
        self.limiter = transfer_limiter() if limiter is _LIMITER_UNSET else limiter
        self.socks, self.inbox, self.outbox, self.writers = {}, {}, {}, []
        self.closed = False
        self.pinned = None
        incoming = [i for i, (a, b) in enumerate(self.links) if b == rank]
        lsock = None
        if incoming:
            lsock = socket.create_server(tuple(addrs[rank]), reuse_port=False)
            lsock.settimeout(timeout_s)
        try:
            # connect every outgoing link (in link order), then accept every incoming one:
            # a connect completes against the peer's listen backlog, so no order deadlocks
            for i, (a, b) in enumerate(self.links):
                if a != rank:
                    continue
                deadline = time.monotonic() + timeout_s
                while True:
                    try:
                        s = socket.create_connection(tuple(addrs[b]), timeout=timeout_s)
                        break
                    except OSError:
                        if time.monotonic() > deadline:
                            raise TimeoutError(f"link {a}->{b}: no listener at {addrs[b]} within {timeout_s} s")
                        time.sleep(0.05)
                s.sendall(struct.pack("<I", i))  # which link this connection carries
                self._attach(i, s, sending=True)
            for _ in incoming:
                s, _ = lsock.accept()
                s.settimeout(timeout_s)
                (i,) = struct.unpack("<I", _read_exact(s, 4))
                if i not in incoming or i in self.socks:
                    raise WireError(f"unexpected link index {i}")
                self._attach(i, s, sending=False)
        finally:
            if lsock is not None:
                lsock.close()

    def _attach(self, i, s, sending):
        s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        s.settimeout(None)
        self.socks[i] = s
        if sending:
            q = queue.Queue()
            self.outbox[i] = q
            th = threading.Thread(target=self._writer, args=(i, s, q), daemon=True)
            self.writers.append(th)
        else:
            q = queue.Queue()
            self.inbox[i] = q
            th = threading.Thread(target=self._reader, args=(i, s, q), daemon=True)
        th.start()

    def _writer(self, i, s, q):
        while True:
            item = q.get()
            if item is None:
                return
            m, fut = item
            try:
                write_message(s, m, self.limiter)
                fut.put(None)
            except Exception as e:  # noqa: BLE001 -- reported to the waiter
                fut.put(e)

    def _reader(self, i, s, q):
        while True:
            try:
                _, m = read_message(s)
            except Exception as e:  # noqa: BLE001 -- reported to the next receive
                q.put(e)
                return
            q.put(m)

    def _next(self, i):
        try:
            m = self.inbox[i].get(timeout=self.timeout_s)
        except queue.Empty:
            raise TimeoutError(f"link {self.links[i]}: no message within {self.timeout_s} s") from None
        if isinstance(m, Exception):
            self.inbox[i].put(m)
            raise WireError(f"link {self.links[i]}: {m}") from m
        return m

    def _link(self, a, b) -> int:
        if (a, b) in self.links:
            return self.links.index((a, b))
        raise ValueError(f"no pipeline link {a} -> {b}")

    def isend(self, t, dst: int):
        i = self._link(self.rank, dst)
        nbytes = t.numel() * t.element_size()
        if t.is_cuda and (self.pinned is None or self.pinned.numel() < nbytes):
            self.pinned = _torch().empty(nbytes, dtype=_torch().uint8, pin_memory=True)
        m = Message.from_tensor(t, pinned=self.pinned if t.is_cuda else None)
        fut = queue.Queue()
        self.outbox[i].put((m, fut))
        return _Sent(fut, self.timeout_s, self.links[i])

    def irecv(self, t, src: int):
        return _Received(self, self._link(src, self.rank), t)

    def close(self) -> None:
        if self.closed:
            return
        self.closed = True
        for q in self.outbox.values():
            q.put(None)
        for th in self.writers:  # the queued frames are written before the sockets close
            th.join(timeout=self.timeout_s)
        for s in self.socks.values():
            try:
                s.shutdown(socket.SHUT_RDWR)
            except OSError:
                pass
            s.close()
        self.socks = {}


# ---------------------------------------------------------------- the master/worker exchange
WORKER_CAPABILITIES = ("compact_batch_v1", "compact_range_batch_v1")  # worker.rs:263-268


def expand_compact_batch(first_layer_name: str, index_pos: int, first_block_idx: int,
                         num_layers: int) -> List[Tuple[str, int, int]]:
    """worker.rs:349-372: the layer names continue the first name's numeric
    suffix, the block indices the first block index."""
    i = len(first_layer_name)
    while i > 0 and first_layer_name[i - 1].isdigit():
        i -= 1
    if i == len(first_layer_name):
        raise WireError("compact batch layer name has no numeric suffix")
    prefix, start = first_layer_name[:i], int(first_layer_name[i:])
    return [(f"{prefix}{start + o}", index_pos, first_block_idx + o) for o in range(num_layers)]


def request_ops(m: Message, names_by_idx) -> List[Tuple[str, int, int]]:
    """The (layer name, index_pos, block index) list a request asks a worker to
    run (worker.rs:661-690); names_by_idx maps the worker's block indices to
    its layer names (for CompactRangeBatch, worker.rs:297-312)."""
    if m.kind == "SingleOp":
        return [(m.layer_name, m.index_pos, m.block_idx)]
    if m.kind == "Batch":
        return [(str(n), int(p), int(b)) for n, p, b in m.batch]
    if m.kind == "CompactBatch":
        b = m.batch
        return expand_compact_batch(b.first_layer_name, b.index_pos, b.first_block_idx, b.num_layers)
    if m.kind == "CompactRangeBatch":
        b = m.batch
        ops = []
        for blk in range(b.first_block_idx, b.first_block_idx + b.num_layers):
            if blk not in names_by_idx:
                raise WireError(f"compact range references missing local block index {blk}")
            ops.append((names_by_idx[blk], b.index_pos, blk))
        return ops
    raise WireError(f"unhandled message in loop: {m.kind}")


class StageWorker:
    """The worker side of the reference's exchange over one connection
    (worker.rs:615-765): a Hello answered with WorkerInfo, then per request
    the layers it names run on its hidden state, answered with a Tensor
    message and the compute time in microseconds.

    run(x, first_block, num_layers, index_pos) computes a contiguous run of
    this worker's blocks at token positions index_pos.. on x (a host tensor in
    the request's dtype and shape) and returns the result (any device).  The
    blocks of one request must be local, contiguous and share one index_pos --
    what the reference's master sends to a worker that holds whole stages."""

    def __init__(self, run, names_by_idx, info: Optional[WorkerInfo] = None):
        self.run, self.names = run, dict(names_by_idx)
        self.info = info or WorkerInfo(version="dial-b200|" + "|".join(WORKER_CAPABILITIES), device="cuda")

    def serve(self, sock, limiter=None) -> int:
        """Serves one connection until the peer closes it; returns the requests served."""
        t0 = time.monotonic()
        _, hello = read_message(sock)
        if hello.kind != "Hello":
            raise WireError(f"unexpected message instead of hello: {hello.kind}")
        self.info.latency = int((time.monotonic() - t0) * 1000)
        write_message(sock, Message("WorkerInfo", info=self.info), limiter)
        served = 0
        while True:
            try:
                _, m = read_message(sock)
            except ConnectionClosed:
                return served
            start = time.monotonic()
            ops = request_ops(m, self.names)
            if not ops:
                raise WireError("request names no layers")
            first, index_pos = ops[0][2], ops[0][1]
            for o, (name, ip, blk) in enumerate(ops):
                if self.names.get(blk) != name:
                    raise WireError(f"could not find layer {name}")
                if ip != index_pos or blk != first + o:
                    raise WireError("a request must name contiguous blocks at one index_pos")
            y = self.run(m.x.to_tensor(), first, len(ops), index_pos)
            us = int((time.monotonic() - start) * 1e6)
            write_message(sock, Message.from_tensor(y, compute_us=us), limiter)
            served += 1


class RemoteStage:
    """The master side (Client::request / forward_batch, client.rs:281-329,
    389-452): connects, sends Hello, reads the worker's WorkerInfo, and sends
    each batch as the most compact message the worker supports -- a
    CompactRangeBatch or CompactBatch when the blocks are contiguous at one
    index_pos, a Batch otherwise."""

    def __init__(self, addr: Tuple[str, int], timeout_s: float = 60.0, limiter=_LIMITER_UNSET):
        self.limiter = transfer_limiter() if limiter is _LIMITER_UNSET else limiter
        self.sock = socket.create_connection(tuple(addr), timeout=timeout_s)
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        write_message(self.sock, Message.hello(), self.limiter)
        _, m = read_message(self.sock)
        if m.kind != "WorkerInfo":
            raise WireError(f"expected WorkerInfo, got {m.kind}")
        self.info = m.info
        self.compact_batch = self.info.supports("compact_batch_v1")
        self.compact_range_batch = self.info.supports("compact_range_batch_v1")
        self.last_compute_us = 0
        self.last_kind = None

    def forward_batch(self, x, batch: Sequence[Tuple[str, int, int]], sampling=None, out=None):
        batch = [(str(n), int(p), int(b)) for n, p, b in batch]
        if not batch:
            raise WireError("empty batch")
        name0, ip0, b0 = batch[0]
        compact = all(p == ip0 for _, p, _ in batch) and all(b == b0 + o for o, (_, _, b) in enumerate(batch))
        rx = RawTensor.from_tensor(x)
        if compact and self.compact_batch and self.compact_range_batch:
            m = Message("CompactRangeBatch", x=rx, batch=CompactRangeBatch(ip0, b0, len(batch)),
                        sampling=sampling)
        elif compact and self.compact_batch:
            m = Message("CompactBatch", x=rx, batch=CompactBatch(name0, ip0, b0, len(batch)), sampling=sampling)
        else:
            m = Message("Batch", x=rx, batch=batch, sampling=sampling)
        self.last_kind = m.kind
        write_message(self.sock, m, self.limiter)
        _, r = read_message(self.sock)
        if r.kind != "Tensor":
            raise WireError(f"expected a Tensor response, got {r.kind}")
        self.last_compute_us = r.compute_us
        return r.x.to_tensor(out=out) if out is not None else r.x.to_tensor()

    def close(self) -> None:
        self.sock.close()

