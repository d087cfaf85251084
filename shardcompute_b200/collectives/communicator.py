"""Communicator: the reference's collective API on NCCL over NVLink.

Drop-in for ``collectives/communicator.py`` of the reference (``Communicator``
:52-603, ``ProcessGroup`` :606-648): same method names, arguments and
semantics (all_reduce sum/mean/max/min, rank-ordered all_gather along any
dim, start/wait_all_reduce, all_reduce_batch, reduce_scatter, broadcast,
barrier, send/recv, stats).  The asyncio-TCP ring / WebSocket-relay
transports of the reference (``collectives/all_reduce.py:58-193``,
``all_gather.py:54-162``, ``point_to_point.py``, ``ws_relay.py``) are replaced
by one NCCL communicator per process, created through ``libsc_b200.so``.

Rendezvous: rank 0 creates the NCCL unique id and publishes it in a
``torch.distributed`` store (a ``TCPStore`` at ``peer_infos[0]`` / the
constructor's host and port, or the default store of an initialised process
group).  Collectives are enqueued on the caller's current CUDA stream, so
they order with the kernels around them and can be captured in CUDA graphs.
``send``/``recv`` are control-plane transfers (small host tensors through the
store), as the reference uses them only to move request metadata.

``backend="gloo"`` runs the same host logic with ``torch.distributed`` on CPU
tensors; it exists so the multi-rank host paths are testable without GPUs.
"""

from __future__ import annotations

import ctypes as C
import datetime
import itertools
import logging
import os
import pickle
import time
from dataclasses import dataclass
from typing import Any, Dict, List, Optional

import torch

logger = logging.getLogger(__name__)

_OPS = {"sum": 0, "max": 1, "min": 2, "mean": 3}

# poll() code for a timed-out NVLink peer-memory collective.
P2P_TIMEOUT = -1
# Communicators a process creates, in order: the same sequence on every rank
# gives matching store keys for each communicator's peer-memory setup.
_P2P_GENERATION = itertools.count()


@dataclass
class CommunicatorStats:
    total_all_reduce_calls: int = 0
    total_all_gather_calls: int = 0
    total_all_reduce_time_ms: float = 0.0
    total_all_gather_time_ms: float = 0.0
    total_bytes_sent: int = 0
    total_bytes_received: int = 0

    def to_dict(self) -> Dict[str, Any]:
        return {
            "total_all_reduce_calls": self.total_all_reduce_calls,
            "total_all_gather_calls": self.total_all_gather_calls,
            "total_all_reduce_time_ms": self.total_all_reduce_time_ms,
            "total_all_gather_time_ms": self.total_all_gather_time_ms,
            "total_bytes_sent": self.total_bytes_sent,
            "total_bytes_received": self.total_bytes_received,
            "avg_all_reduce_time_ms": (self.total_all_reduce_time_ms / self.total_all_reduce_calls
                                       if self.total_all_reduce_calls else 0),
            "avg_all_gather_time_ms": (self.total_all_gather_time_ms / self.total_all_gather_calls
                                       if self.total_all_gather_calls else 0),
        }


class Communicator:
    """Collectives for tensor parallelism (one process per GPU)."""

    def __init__(self, rank: int, world_size: int, host: str = "127.0.0.1", port: int = 9000,
                 topology_type: str = "ring", backend: str = "nccl"):
        if backend not in ("nccl", "gloo"):
            raise ValueError(f"backend must be 'nccl' or 'gloo', got {backend}")
        self.rank = rank
        self.world_size = world_size
        self.host = host
        self.port = port
        self.topology_type = topology_type  # accepted for compatibility; NCCL picks its own algorithm
        self.backend = backend
        self.stats = CommunicatorStats()
        self._initialized = False
        self._comm = None  # opaque sc_comm handle (nccl backend)
        self._store = None
        self._pg = None  # torch.distributed group (gloo backend)
        self._pending: Dict[str, Any] = {}
        self._ar_counter = 0
        self._barrier_counter = 0
        self._bcast_counter = 0
        self._p2p_counter: Dict[tuple, int] = {}
        self._comm_stream: Optional[torch.cuda.Stream] = None
        self._p2p = None  # sc_p2p handle: NVLink one-shot collectives for small messages
        self._p2p_max = 0
        self._extra_arenas: List[tuple] = []  # (handle, store prefix) of arenas lent to kernels

    # ------------------------------------------------------------ setup

    @property
    def is_initialized(self) -> bool:
        return self._initialized

    async def initialize(self, peer_infos: Optional[List[Any]] = None, timeout: float = 30.0, store=None):
        """Rendezvous and create the communicator.

        ``peer_infos`` (reference ``PeerInfo`` list) only supplies rank 0's
        host/port for the store; ``store`` may be given directly instead.
        """
        self.initialize_sync(peer_infos=peer_infos, timeout=timeout, store=store)

    def initialize_sync(self, peer_infos=None, timeout: float = 30.0, store=None):
        if self._initialized:
            logger.warning("Communicator already initialized")
            return
        import torch.distributed as dist

        if store is None and dist.is_available() and dist.is_initialized():
            store = dist.distributed_c10d._get_default_store()
        if store is None:
            host, port = self.host, self.port
            if peer_infos:
                p0 = peer_infos[0]
                host = getattr(p0, "host", host)
                port = getattr(p0, "port", port)
            store = dist.TCPStore(host, port, self.world_size, self.rank == 0,
                                  timeout=datetime.timedelta(seconds=timeout))
        self._store = store
        if self.backend == "gloo":
            if not dist.is_initialized():
                dist.init_process_group("gloo", store=store, rank=self.rank, world_size=self.world_size,
                                        timeout=datetime.timedelta(seconds=timeout))
            self._pg = dist.group.WORLD
        else:
            from .. import _lib as L

            lib = L.load()
            uid = (C.c_char * 128)()
            key = "shardcompute_b200/nccl_uid"
            if self.rank == 0:
                L.check(lib.sc_comm_unique_id(uid, 128), "sc_comm_unique_id")
                store.set(key, bytes(uid))
            else:
                store.wait([key], datetime.timedelta(seconds=timeout))
                C.memmove(uid, store.get(key), 128)
            handle = C.c_void_p()
            L.check(lib.sc_comm_init(uid, 128, self.world_size, self.rank, C.byref(handle)), "sc_comm_init")
            self._comm = handle
            self._comm_stream = torch.cuda.Stream()
            self._init_p2p(timeout)
        self._initialized = True

    def _init_p2p(self, timeout: float):
        """Map every peer's IPC arena for the NVLink one-shot collectives.

        Used for all-reduce (sum, f16/f32) and all-gather (4-byte types) of
        messages up to ``SC_P2P_MAX_BYTES`` (default 1 MiB); ``SC_P2P=0``
        keeps everything on NCCL.  Ranks publish whether their setup worked
        and either all use the transport or none does."""
        gen = next(_P2P_GENERATION)
        if self.world_size < 2 or self.world_size > 8 or os.environ.get("SC_P2P", "1") == "0":
            return
        max_bytes = int(os.environ.get("SC_P2P_MAX_BYTES", 1 << 20))
        handle = self._open_arena(f"shardcompute_b200/p2p/{gen}", max_bytes, timeout)
        if handle is not None:
            self._p2p, self._p2p_max = handle, max_bytes
            self._p2p_gen = gen

    def _open_arena(self, pre: str, max_bytes: int, timeout: float):
        """Collective: create this rank's peer-memory arena, exchange IPC
        handles through the store, map every peer's.  Returns the transport
        handle when every rank succeeded, else None on every rank."""
        from .. import _lib as L

        lib = L.load()
        hb = int(lib.sc_p2p_handle_bytes())
        handle = C.c_void_p()
        buf = (C.c_char * hb)()
        ok = lib.sc_p2p_create(self.world_size, self.rank, max_bytes, C.byref(handle), buf, hb) == L.SC_OK
        if not ok:
            logger.warning("p2p transport unavailable on rank %d: %s", self.rank, L.last_error())
        wait = datetime.timedelta(seconds=timeout)
        self._store.set(f"{pre}/h/{self.rank}", bytes(buf) if ok else b"-")
        keys = [f"{pre}/h/{q}" for q in range(self.world_size)]
        self._store.wait(keys, wait)
        hs = [self._store.get(k) for k in keys]
        if ok and all(len(h) == hb for h in hs):
            table = (C.c_char * (hb * self.world_size))()
            for q, h in enumerate(hs):
                C.memmove(C.addressof(table) + q * hb, h, hb)
            ok = lib.sc_p2p_open(handle, table, hb) == L.SC_OK
            if not ok:
                logger.warning("p2p open failed on rank %d: %s", self.rank, L.last_error())
        else:
            ok = False
        self._store.set(f"{pre}/ok/{self.rank}", b"1" if ok else b"0")
        keys = [f"{pre}/ok/{q}" for q in range(self.world_size)]
        self._store.wait(keys, wait)
        if all(self._store.get(k) == b"1" for k in keys):
            return handle
        if handle.value:
            lib.sc_p2p_destroy(handle)
        return None

    def step_arena(self, nbytes: int, timeout: float = 60.0):
        """Collective: a dedicated peer-memory arena of at least ``nbytes``
        per rank for a kernel that lays out its own lines (the persistent
        decode step), returned as (every rank's arena base as mapped here,
        arena bytes).  Freed at shutdown.  Raises if any rank failed."""
        from .. import _lib as L

        self._require()
        gen = next(_P2P_GENERATION)
        pre = f"shardcompute_b200/step_arena/{gen}"
        # an arena is a 4 KB header + 2 x world regions of 16-byte lines per 8 payload bytes
        max_bytes = max(8, -(-max(0, nbytes - 4096) // (4 * self.world_size)) + 16)
        handle = self._open_arena(pre, max_bytes, timeout)
        if handle is None:
            raise RuntimeError(f"rank {self.rank}: the decode step's peer-memory arena could not be set up")
        bases = (C.c_void_p * self.world_size)()
        size = C.c_size_t()
        L.check(L.load().sc_p2p_arenas(handle, C.cast(bases, L._pp), C.byref(size)), "sc_p2p_arenas")
        if size.value < nbytes:
            raise RuntimeError(f"step arena of {size.value} bytes < {nbytes}")
        self._extra_arenas.append((handle, pre))
        return [bases[q] for q in range(self.world_size)], size.value

    def fused_transport(self, max_bytes: int, timeout: float = 60.0):
        """Collective: a dedicated peer-memory transport (a handle for
        ``sc_qlinear_allreduce``) carrying messages of up to ``max_bytes``
        per rank, freed at shutdown; None on every rank when any rank failed
        (the caller then keeps the GEMV + all-reduce pair).  Its per-CTA
        epochs live in its own header, so no other collective shares it."""
        self._require()
        if self.world_size < 2 or self.world_size > 8 or self.backend != "nccl":
            return None
        gen = next(_P2P_GENERATION)
        pre = f"shardcompute_b200/fused_ar/{gen}"
        handle = self._open_arena(pre, max(8, int(max_bytes)), timeout)
        if handle is None:
            return None
        self._extra_arenas.append((handle, pre))
        return handle

    @property
    def p2p_enabled(self) -> bool:
        """True when small all-reduces / all-gathers go through NVLink peer memory."""
        return self._p2p is not None

    def _p2p_fits(self, t: torch.Tensor, dtypes) -> bool:
        return (self._p2p is not None and t.dtype in dtypes
                and t.numel() * t.element_size() <= self._p2p_max)

    def _require(self):
        if not self._initialized:
            raise RuntimeError("Communicator not initialized")

    def _device(self) -> torch.device:
        return torch.device("cpu") if self.backend == "gloo" else torch.device("cuda", torch.cuda.current_device())

    # ------------------------------------------------------------ raw NCCL (engine path)

    def _dt(self, t: torch.Tensor) -> int:
        from .. import _lib as L

        return {torch.float16: L.SC_F16, torch.float32: L.SC_F32, torch.int32: L.SC_I32}[t.dtype]

    def allreduce_into(self, send: torch.Tensor, recv: torch.Tensor, op: str = "sum") -> None:
        """Enqueue an all-reduce of ``send`` into ``recv`` on the current stream (graph-capturable)."""
        self._require()
        if op not in _OPS:
            raise ValueError(f"Unknown reduction op: {op}")
        if self.world_size == 1:
            if recv.data_ptr() != send.data_ptr():
                recv.copy_(send)
            return
        if self.backend == "gloo":
            import torch.distributed as dist

            buf = send.clone()
            dist.all_reduce(buf, op=_gloo_op(op), group=self._pg)
            if op == "mean":
                buf /= self.world_size
            recv.copy_(buf)
            return
        from .. import _lib as L

        stream = torch.cuda.current_stream(send.device).cuda_stream
        if op == "sum" and self._p2p_fits(send, (torch.float16, torch.float32)):
            L.call("sc_p2p_allreduce", send.data_ptr(), recv.data_ptr(), send.numel(), self._dt(send), self._p2p,
                   stream)
            return
        L.call("sc_allreduce", send.data_ptr(), recv.data_ptr(), send.numel(), self._dt(send), _OPS[op],
               self._comm, stream)

    def allgather_into(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        """Enqueue an all-gather: ``recv`` is ``[world, *send.shape]`` contiguous."""
        self._require()
        if self.world_size == 1:
            recv.view_as(send).copy_(send)
            return
        if self.backend == "gloo":
            import torch.distributed as dist

            parts = [torch.empty_like(send) for _ in range(self.world_size)]
            dist.all_gather(parts, send.contiguous(), group=self._pg)
            recv.copy_(torch.stack(parts))
            return
        from .. import _lib as L

        stream = torch.cuda.current_stream(send.device).cuda_stream
        if self._p2p_fits(send, (torch.float32, torch.int32)):
            L.call("sc_p2p_allgather", send.data_ptr(), recv.data_ptr(), send.numel(), self._dt(send), self._p2p,
                   stream)
            return
        L.call("sc_allgather", send.data_ptr(), recv.data_ptr(), send.numel(), self._dt(send), self._comm, stream)

    # ------------------------------------------------------------ reference API

    def _reduce_tensor(self, tensor: torch.Tensor, op: str) -> torch.Tensor:
        if op not in _OPS:
            raise ValueError(f"Unknown reduction op: {op}")
        src = tensor.contiguous()
        out = torch.empty_like(src)
        self.allreduce_into(src, out, op)
        return out

    async def all_reduce(self, tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
        self._require()
        t0 = time.perf_counter()
        out = self._reduce_tensor(tensor, op)
        self.stats.total_all_reduce_calls += 1
        self.stats.total_all_reduce_time_ms += (time.perf_counter() - t0) * 1000
        nb = tensor.numel() * tensor.element_size() * (self.world_size - 1) * 2 // max(self.world_size, 1)
        self.stats.total_bytes_sent += nb
        self.stats.total_bytes_received += nb
        return out

    def start_all_reduce(self, tensor: torch.Tensor, op: str = "sum") -> str:
        """Non-blocking all-reduce on the comm stream; the id is redeemed by wait_all_reduce."""
        self._require()
        self._ar_counter += 1
        op_id = f"ar_{self.rank}_{self._ar_counter}"
        if self.backend == "gloo" or self.world_size == 1:
            self._pending[op_id] = (self._reduce_tensor(tensor, op), None, time.perf_counter())
            return op_id
        cur = torch.cuda.current_stream(tensor.device)
        src = tensor.contiguous()
        out = torch.empty_like(src)
        self._comm_stream.wait_stream(cur)
        with torch.cuda.stream(self._comm_stream):
            self.allreduce_into(src, out, op)
            ev = torch.cuda.Event()
            ev.record(self._comm_stream)
        src.record_stream(self._comm_stream)
        out.record_stream(self._comm_stream)
        self._pending[op_id] = (out, ev, time.perf_counter())
        return op_id

    async def wait_all_reduce(self, op_id: str) -> torch.Tensor:
        if op_id not in self._pending:
            raise ValueError(f"Unknown all-reduce operation ID: {op_id}")
        out, ev, t0 = self._pending.pop(op_id)
        if ev is not None:
            torch.cuda.current_stream(out.device).wait_event(ev)
        self.stats.total_all_reduce_calls += 1
        self.stats.total_all_reduce_time_ms += (time.perf_counter() - t0) * 1000
        return out

    async def all_reduce_batch(self, tensors: List[torch.Tensor], op: str = "sum") -> List[torch.Tensor]:
        """One all-reduce over the concatenation of ``tensors`` (counted as one call)."""
        self._require()
        if not tensors:
            return []
        if len(tensors) == 1:
            return [await self.all_reduce(tensors[0], op)]
        dtype = tensors[0].dtype
        if any(t.dtype != dtype for t in tensors):
            raise ValueError("All tensors must have same dtype for batched all-reduce")
        red = await self.all_reduce(torch.cat([t.reshape(-1) for t in tensors]), op)
        outs, off = [], 0
        for t in tensors:
            outs.append(red[off:off + t.numel()].view(t.shape))
            off += t.numel()
        return outs

    async def all_gather(self, tensor: torch.Tensor, dim: int = -1) -> torch.Tensor:
        """Rank-ordered concatenation along ``dim`` (reference all_gather.py:90-162)."""
        self._require()
        if self.world_size == 1:
            return tensor
        t0 = time.perf_counter()
        src = tensor.contiguous()
        buf = torch.empty((self.world_size, *src.shape), dtype=src.dtype, device=src.device)
        self.allgather_into(src, buf)
        d = dim if dim >= 0 else src.dim() + dim
        out = torch.cat(list(buf.unbind(0)), dim=d)
        self.stats.total_all_gather_calls += 1
        self.stats.total_all_gather_time_ms += (time.perf_counter() - t0) * 1000
        nb = src.numel() * src.element_size() * (self.world_size - 1)
        self.stats.total_bytes_sent += nb
        self.stats.total_bytes_received += nb
        return out

    async def reduce_scatter(self, tensor: torch.Tensor, op: str = "sum", dim: int = -1) -> torch.Tensor:
        """Reduce across ranks; return this rank's 1/N slice along ``dim``."""
        self._require()
        red = self._reduce_tensor(tensor, op)
        d = dim if dim >= 0 else red.dim() + dim
        return red.chunk(self.world_size, dim=d)[self.rank].contiguous()

    async def broadcast(self, tensor: Optional[torch.Tensor], root: int = 0) -> torch.Tensor:
        """Root's tensor on every rank; non-roots may pass None (shape/dtype travel via the store)."""
        self._require()
        self._bcast_counter += 1
        key = f"shardcompute_b200/bcast/{self._bcast_counter}"
        if self.rank == root:
            if tensor is None:
                raise ValueError("Root must provide tensor for broadcast")
            if self.world_size > 1:
                self._store.set(key, pickle.dumps((tuple(tensor.shape), str(tensor.dtype))))
            src = tensor.contiguous()
        else:
            self._store.wait([key], datetime.timedelta(seconds=60))
            shape, dt = pickle.loads(self._store.get(key))
            src = torch.empty(shape, dtype=getattr(torch, dt.split(".")[-1]), device=self._device())
        if self.world_size == 1:
            return src
        if self.backend == "gloo":
            import torch.distributed as dist

            dist.broadcast(src, src=root, group=self._pg)
            return src
        from .. import _lib as L

        L.call("sc_broadcast", src.data_ptr(), src.data_ptr(), src.numel(), self._dt(src), root, self._comm,
               torch.cuda.current_stream(src.device).cuda_stream)
        return src

    async def barrier(self):
        self._require()
        self._barrier_counter += 1
        dev = self._device()
        t = torch.tensor([float(self._barrier_counter)], dtype=torch.float32, device=dev)
        await self.all_reduce(t, op="sum")
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()

    def _nccl_p2p(self, tensor: Optional[torch.Tensor] = None) -> bool:
        return (self.backend != "gloo" and self._comm is not None and
                (tensor is None or tensor.device.type == "cuda"))

    def send_into(self, tensor: torch.Tensor, dest: int) -> None:
        """Enqueue a send of ``tensor``'s bytes to ``dest`` on the current
        stream (NCCL; graph-capturable).  ``dest`` must post a matching
        ``recv_into`` of the same byte count."""
        self._require()
        if dest == self.rank or not 0 <= dest < self.world_size:
            raise ValueError(f"Invalid destination rank: {dest}")
        if not self._nccl_p2p(tensor):
            raise RuntimeError("send_into needs the NCCL backend and a CUDA tensor")
        from .. import _lib as L

        t = tensor.contiguous()
        L.call("sc_send", t.data_ptr(), t.numel() * t.element_size(), L.SC_U8, dest, self._comm,
               torch.cuda.current_stream(t.device).cuda_stream)
        self.stats.total_bytes_sent += t.numel() * t.element_size()

    def recv_into(self, tensor: torch.Tensor, source: int) -> torch.Tensor:
        """Enqueue a receive from ``source`` into ``tensor`` (contiguous, the
        sender's byte count) on the current stream (NCCL; graph-capturable)."""
        self._require()
        if source == self.rank or not 0 <= source < self.world_size:
            raise ValueError(f"Invalid source rank: {source}")
        if not self._nccl_p2p(tensor) or not tensor.is_contiguous():
            raise RuntimeError("recv_into needs the NCCL backend and a contiguous CUDA tensor")
        from .. import _lib as L

        L.call("sc_recv", tensor.data_ptr(), tensor.numel() * tensor.element_size(), L.SC_U8, source, self._comm,
               torch.cuda.current_stream(tensor.device).cuda_stream)
        self.stats.total_bytes_received += tensor.numel() * tensor.element_size()
        return tensor

    async def send(self, tensor: torch.Tensor, dest: int):
        """Point-to-point send (collectives/communicator.py:520-541).  CUDA
        tensors on the NCCL backend: the shape and dtype go through the store,
        the bytes through NCCL on the current stream.  Otherwise the whole
        tensor goes through the store (control plane, CPU tests)."""
        self._require()
        if dest == self.rank or not 0 <= dest < self.world_size:
            raise ValueError(f"Invalid destination rank: {dest}")
        n = self._p2p_counter.get((self.rank, dest), 0) + 1
        self._p2p_counter[(self.rank, dest)] = n
        key = f"shardcompute_b200/p2p/{self.rank}->{dest}/{n}"
        if self._nccl_p2p(tensor):
            self._store.set(key, pickle.dumps((tuple(tensor.shape), str(tensor.dtype), None)))
            self.send_into(tensor, dest)
            return
        self._store.set(key, pickle.dumps((tuple(tensor.shape), str(tensor.dtype),
                                           tensor.detach().cpu().contiguous().numpy().tobytes())))

    async def recv(self, source: int) -> torch.Tensor:
        """Point-to-point receive of the next tensor ``source`` sent to this
        rank (collectives/communicator.py:543-561)."""
        self._require()
        if source == self.rank or not 0 <= source < self.world_size:
            raise ValueError(f"Invalid source rank: {source}")
        import numpy as np

        n = self._p2p_counter.get((source, self.rank), 0) + 1
        self._p2p_counter[(source, self.rank)] = n
        key = f"shardcompute_b200/p2p/{source}->{self.rank}/{n}"
        self._store.wait([key], datetime.timedelta(seconds=60))
        shape, dt, raw = pickle.loads(self._store.get(key))
        if raw is None:  # the bytes travel through NCCL
            t = torch.empty(shape, dtype=getattr(torch, dt.split(".")[-1]), device=self._device())
            return self.recv_into(t, source)
        t = torch.from_numpy(np.frombuffer(bytearray(raw), dtype=_np_dtype(dt)).reshape(shape).copy())
        return t.to(self._device())

    def flush_peers(self):
        """NCCL keeps no per-peer receive queues; nothing to discard."""
        return None

    def get_stats(self) -> Dict[str, Any]:
        return self.stats.to_dict()

    def reset_stats(self):
        self.stats = CommunicatorStats()

    # ------------------------------------------------------------ failure handling

    def poll(self) -> int:
        """0 when healthy, else NCCL's asynchronous error code, or
        ``P2P_TIMEOUT`` when a peer-memory collective gave up waiting for a
        peer.  Never blocks and makes no GPU call."""
        if self.backend != "nccl" or self._comm is None:
            return 0
        from .. import _lib as L

        # the collectives' transport and those lent to kernels (the fused
        # GEMV all-reduce raises the same sticky word on a timeout)
        for h in ([self._p2p] if self._p2p is not None else []) + [a[0] for a in self._extra_arenas]:
            t = C.c_int(0)
            L.check(L.load().sc_p2p_status(h, C.byref(t)), "sc_p2p_status")
            if t.value:
                return P2P_TIMEOUT
        err = C.c_int(0)
        L.check(L.load().sc_comm_poll(self._comm, C.byref(err)), "sc_comm_poll")
        return err.value

    def check_health(self):
        """Raise if a collective failed (TimeoutError for a peer that stopped
        answering a peer-memory collective, RuntimeError for NCCL)."""
        code = self.poll()
        if code == P2P_TIMEOUT:
            raise TimeoutError(f"rank {self.rank}: a peer-memory collective timed out waiting for a peer")
        if code:
            raise RuntimeError(f"rank {self.rank}: NCCL asynchronous error {code}")

    def _close_p2p(self, wait_for_peers: bool):
        """Free the peer-memory transports; first (unless aborting) wait until
        every rank got here, so no peer still sends into this rank's arenas."""
        from .. import _lib as L

        arenas = list(self._extra_arenas)
        if self._p2p is not None:
            arenas.append((self._p2p, f"shardcompute_b200/p2p/{self._p2p_gen}"))
        if not arenas:
            return
        if wait_for_peers:
            pre = arenas[-1][1]
            self._store.set(f"{pre}/bye/{self.rank}", b"1")
            try:
                self._store.wait([f"{pre}/bye/{q}" for q in range(self.world_size)], datetime.timedelta(seconds=60))
            except Exception:  # noqa: BLE001 - a dead peer sends nothing more
                logger.warning("rank %d: peers missing at p2p shutdown", self.rank)
        for handle, _ in arenas:
            L.load().sc_p2p_destroy(handle)
        self._extra_arenas = []
        self._p2p = None

    def abort(self):
        """Tear the communicator down without waiting for peers (unblocks a rank stuck on a dead peer)."""
        if self.backend == "nccl" and self._comm is not None:
            self._close_p2p(wait_for_peers=False)
            from .. import _lib as L

            L.load().sc_comm_abort(self._comm)
            self._comm = None
        self._initialized = False

    async def shutdown(self):
        self.shutdown_sync()

    def shutdown_sync(self):
        if self.backend == "nccl" and self._comm is not None:
            from .. import _lib as L

            torch.cuda.synchronize()
            self._close_p2p(wait_for_peers=True)
            L.check(L.load().sc_comm_destroy(self._comm), "sc_comm_destroy")
            self._comm = None
        self._initialized = False


def _gloo_op(op: str):
    import torch.distributed as dist

    if op not in _OPS:
        raise ValueError(f"Unknown reduction op: {op}")
    return {"sum": dist.ReduceOp.SUM, "mean": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX,
            "min": dist.ReduceOp.MIN}[op]


def _np_dtype(torch_dtype_str: str):
    import numpy as np

    name = torch_dtype_str.split(".")[-1]
    return {"float16": np.float16, "float32": np.float32, "float64": np.float64, "int32": np.int32,
            "int64": np.int64, "uint8": np.uint8}[name]


class ProcessGroup:
    """Subgroup wrapper; like the reference it proxies the full communicator."""

    def __init__(self, ranks: List[int], local_rank: int, comm: Communicator):
        self.ranks = ranks
        self.local_rank = local_rank
        self.size = len(ranks)
        self.comm = comm
        self.group_to_global = {i: r for i, r in enumerate(ranks)}
        self.global_to_group = {r: i for i, r in enumerate(ranks)}
        self.group_rank = self.global_to_group[local_rank]

    async def all_reduce(self, tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
        return await self.comm.all_reduce(tensor, op)

    async def all_gather(self, tensor: torch.Tensor, dim: int = -1) -> torch.Tensor:
        return await self.comm.all_gather(tensor, dim)
