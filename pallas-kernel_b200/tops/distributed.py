"""Multi-GPU helpers for the GLA ops (one process per GPU, ``torch.distributed``).

The reference has no multi-device code; BASELINE asks for two layouts:

* **batch x heads sharding** (configs 2 and 3): the (sequence, head) units are
  independent, so every rank runs the ops on its own slice with no collective.
  :func:`shard` picks a rank's slice.

* **sequence parallelism** (config 4): one long sequence is split into contiguous
  spans, one per rank.  The chunked scan is linear in the incoming state
  (tops/ops/common/chunk_h.py:372-386): a span's final state is
  ``D * H_in + S`` with ``S`` its final state from a zero state and
  ``D = exp(sum of its gates)`` (diagonal in K).  Each rank computes ``(S, D)``,
  the ranks all-gather them, every rank forms its incoming state ``H_r`` by a
  prefix over the earlier ranks, then runs the full forward with ``H_r``.  The
  backward is the transpose: ``dH_r = D_r * dH_{r+1} + dh0_local_r``, gathered
  and combined as a suffix.  The forward is exact (the same linear algebra the
  single-device scan does), so concatenating the ranks' outputs equals the
  single-device result.

The compute steps are passed in as callables so that the exchange logic can be
tested on CPU ranks (gloo) with any implementation of the local ops; the GPU
defaults use this library's kernels.
"""
from __future__ import annotations

import ctypes
import threading
import time
from typing import Callable

import torch
import torch.distributed as dist

__all__ = ["shard", "prefix_states", "suffix_grads", "all_gather_stack", "seq_parallel_forward",
           "seq_parallel_backward", "seq_parallel_forward_phased", "seq_parallel_backward_phased",
           "chunk_gla_seq_parallel", "NcclStateExchange", "P2PStateExchange", "PeerWatchdog", "PeerLostError"]


class PeerLostError(RuntimeError):
    """A rank of the group left, crashed or stalled: detected on the host before a collective."""


class PeerWatchdog:
    """Host-side liveness of every rank of a group, through the group's key-value store.

    A daemon thread publishes this rank's heartbeat (a counter) every ``interval`` seconds and
    reads the other ranks'.  A peer whose heartbeat has not advanced for ``timeout`` seconds,
    that announced it left (:meth:`close`), or whose store became unreachable marks the group
    lost; :meth:`check` (no I/O) then raises :class:`PeerLostError`.  The exchange calls it
    before it launches a collective, so a rank never enqueues NCCL work that would wait on
    the GPU for a peer that is gone.  ``store`` defaults to the default process group's store.
    """

    def __init__(self, store=None, rank=None, world=None, timeout: float = 30.0, interval: float = 0.2,
                 prefix: str = "tops_gla/heartbeat"):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = dist.PrefixStore(prefix, store)
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.timeout, self.interval = float(timeout), float(interval)
        self.lost: str | None = None
        self._stop = threading.Event()
        now = time.monotonic()
        self._last = {r: None for r in range(self.world) if r != self.rank}
        self._seen = {r: now for r in self._last}
        self.store.set(str(self.rank), "0")
        self._thread = threading.Thread(target=self._run, name="tops-gla-peer-watchdog", daemon=True)
        self._thread.start()

    def _poll(self, beat: int) -> None:
        self.store.set(str(self.rank), str(beat))
        now = time.monotonic()
        for r in self._last:
            key = str(r)
            v = self.store.get(key) if self.store.check([key]) else None
            if v == b"left":
                self.lost = f"rank {r} left the group"
            elif v is not None and v != self._last[r]:
                self._last[r], self._seen[r] = v, now
            elif now - self._seen[r] > self.timeout:
                self.lost = f"rank {r} sent no heartbeat for {now - self._seen[r]:.1f} s"

    def _run(self) -> None:
        beat = 1
        while not self._stop.wait(self.interval) and self.lost is None:
            try:
                self._poll(beat)
            except Exception as e:  # the store itself is gone (its host rank died)
                self.lost = f"the group's store is unreachable ({type(e).__name__}: {e})"
            beat += 1

    def check(self) -> None:
        """Raise PeerLostError if a peer is known to be gone (no I/O)."""
        if self.lost is not None:
            raise PeerLostError(f"rank {self.rank}: {self.lost}")

    def close(self) -> None:
        """Stop the thread and tell the other ranks that this one leaves."""
        self._stop.set()
        self._thread.join(timeout=max(1.0, 5 * self.interval))
        try:
            self.store.set(str(self.rank), "left")
        except Exception:
            pass


class NcclStateExchange:
    """The C ABI's state exchange (``tops_gla_state_exchange``: one ncclAllGather of the
    packed (state, decay) pairs and one prefix / suffix kernel) on a communicator of this
    library's own; ``group`` only broadcasts NCCL's unique id.  Every rank of the group must
    construct it (communicator creation is collective).

    Failure handling: with ``liveness_timeout`` (seconds; None turns it off) a
    :class:`PeerWatchdog` tracks the other ranks on the host, and every exchange first checks
    it: if a peer left or stalled, the communicator is aborted (``tops_gla_nccl_comm_abort``,
    which does not wait for peers) and :class:`PeerLostError` is raised before any NCCL work is
    enqueued.  :meth:`wait` bounds the host's wait for an exchange already launched."""

    _made = 0

    def __init__(self, group=None, liveness_timeout: float | None = 30.0):
        from . import _C
        self._C = _C
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.watchdog = None
        idbuf = (ctypes.c_char * 128)()
        if self.rank == 0:
            _C.call("tops_gla_nccl_get_unique_id", ctypes.addressof(idbuf))
        obj = [bytes(idbuf)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        ctypes.memmove(idbuf, obj[0], 128)
        self.comm = ctypes.c_void_p()
        _C.call("tops_gla_nccl_comm_init", ctypes.byref(self.comm), self.world, ctypes.addressof(idbuf), self.rank)
        NcclStateExchange._made += 1  # the same count on every rank: construction is collective
        if liveness_timeout is not None and group is None:
            self.watchdog = PeerWatchdog(timeout=liveness_timeout, prefix=f"tops_gla/exchange{NcclStateExchange._made}")

    def check_peers(self) -> None:
        """Raise PeerLostError (after aborting the communicator) if a peer is gone."""
        if self.watchdog is None:
            return
        try:
            self.watchdog.check()
        except PeerLostError:
            self.abort()
            raise

    def abort(self) -> None:
        """Abort the communicator without waiting for peers (the handle is freed)."""
        if self.comm:
            self._C.lib().tops_gla_nccl_comm_abort(self.comm)
            self.comm = ctypes.c_void_p()
        if self.watchdog is not None:
            self.watchdog.close()
            self.watchdog = None

    def wait(self, timeout_s: float, stream=None) -> None:
        """Wait on the host, at most ``timeout_s``, for the exchanges enqueued so far; on an NCCL
        error or at the deadline the communicator is aborted and TopsError is raised."""
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        self._C.call("tops_gla_state_exchange_wait", self.comm, st, max(1, int(timeout_s * 1000)))

    def _run(self, backward: bool, local: torch.Tensor, decay: torch.Tensor, boundary, want_total: bool):
        C = self._C
        self.check_peers()
        if not self.comm:
            raise PeerLostError("the exchange's communicator was aborted")
        local = local.float().contiguous()
        decay = decay.float().contiguous()
        boundary = None if boundary is None else boundary.float().contiguous()
        N, H, K, V = local.shape
        out = torch.empty_like(local)
        total = torch.empty_like(local) if want_total else None
        a = C.ExchangeArgs(self.comm, self.rank, self.world, N, H, K, V, int(backward), C.ptr(local), C.ptr(decay),
                           C.ptr(boundary), C.ptr(out), C.ptr(total), None, 0)
        n = int(C.lib().tops_gla_state_exchange_workspace_size(a))
        ws = torch.empty(n, dtype=torch.uint8, device=local.device)
        a.workspace, a.workspace_bytes = C.ptr(ws), n
        C.call("tops_gla_state_exchange", a, C.stream_of(local))
        return out, total

    def forward(self, S, D, h0=None):
        """-> (this rank's incoming state, the whole sequence's final state)."""
        return self._run(False, S, D, h0, True)

    def backward(self, L, D, dht=None):
        """-> the final-state gradient this rank's backward must use."""
        return self._run(True, L, D, dht, False)[0]

    def close(self):
        if self.comm:
            self._C.call("tops_gla_nccl_comm_destroy", self.comm)
            self.comm = ctypes.c_void_p()
        if self.watchdog is not None:
            self.watchdog.close()
            self.watchdog = None


class P2PStateExchange:
    """The state exchange through peer memory (``tops_gla_p2p_exchange``): every rank's
    packed (state, decay) goes straight into its slot of every rank's receive region over
    NVLink, an epoch flag follows, and each rank folds the prefix / suffix from its own region
    once every rank's flag has arrived -- two kernels, no NCCL launch, bit-identical to
    :class:`NcclStateExchange`.  One process per GPU of one host; every rank of the group must
    construct it and run the same exchanges in the same order (as with any collective).

    A region per (N, H, K, V) is allocated on first use (collectively: IPC handles are
    exchanged through the group, then every rank maps every region), so the first exchange of
    a shape must not be inside a CUDA-graph capture; later ones can be captured and replayed
    (the epoch lives in device memory).  Failure handling: the same host-side
    :class:`PeerWatchdog` check before every exchange as NcclStateExchange, and the device-side
    wait for a peer's flag gives up after ``timeout_s`` (device error 3, output not written)."""

    _made = 0

    def __init__(self, group=None, liveness_timeout: float | None = 30.0, timeout_s: float = 10.0,
                 fused: bool = True):
        import socket

        from . import _C
        self._C = _C
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.timeout_ms = max(1, int(timeout_s * 1000))
        where = [None] * self.world
        dist.all_gather_object(where, (socket.gethostname(), str(torch.cuda.get_device_properties(self.device).uuid)),
                               group=group)
        if len({h for h, _ in where}) != 1 or len({u for _, u in where}) != self.world:
            raise ValueError("P2PStateExchange needs one process per GPU on one host (use NcclStateExchange)")
        self.regions = {}  # (N, H, K, V) -> (own region, [mapped peer regions], device table of all)
        # chunk_gla_seq_parallel lets the span kernels that compute a rank's state push it into
        # the regions themselves (tops_gla_chunk_{fwd,bwd}_span_begin_p2p + tops_gla_p2p_combine)
        self.fused_push = bool(fused)
        self.watchdog = None
        P2PStateExchange._made += 1
        if liveness_timeout is not None and group is None:
            self.watchdog = PeerWatchdog(timeout=liveness_timeout, prefix=f"tops_gla/p2p{P2PStateExchange._made}")

    def _args(self, shape, backward=0):
        N, H, K, V = shape
        return self._C.P2PArgs(self.rank, self.world, N, H, K, V, int(backward), None, None, None, None, None, None,
                               None, self.timeout_ms)

    def _region(self, shape):
        reg = self.regions.get(shape)
        if reg is not None:
            return reg
        C, L = self._C, self._C.lib()
        own, mapped, handle, err = ctypes.c_void_p(), [], None, None
        try:
            nbytes = int(L.tops_gla_p2p_region_size(ctypes.byref(self._args(shape))))
            C.call("tops_gla_p2p_alloc", nbytes, ctypes.byref(own))
            hbuf = (ctypes.c_char * C.IPC_HANDLE_BYTES)()
            C.call("tops_gla_ipc_handle", own, ctypes.addressof(hbuf))
            handle = bytes(hbuf)
        except Exception as e:  # noqa: BLE001 -- every rank must learn of it before going on
            err = f"{type(e).__name__}: {e}"
        handles = [None] * self.world
        dist.all_gather_object(handles, (handle, err), group=self.group)
        ptrs = []
        if all(h is not None for h, _ in handles):
            try:
                for j, (hb, _) in enumerate(handles):
                    if j == self.rank:
                        ptrs.append(own.value)
                        continue
                    buf = (ctypes.c_char * C.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                    pj = ctypes.c_void_p()
                    C.call("tops_gla_ipc_open", ctypes.addressof(buf), ctypes.byref(pj))
                    mapped.append(pj)
                    ptrs.append(pj.value)
            except Exception as e:  # noqa: BLE001
                err = f"{type(e).__name__}: {e}"
        outcome = [None] * self.world
        dist.all_gather_object(outcome, err, group=self.group)
        failed = [(j, e) for j, e in enumerate(outcome) if e is not None]
        if failed:  # every rank unwinds and raises together, so their collectives stay paired
            for pj in mapped:
                C.lib().tops_gla_ipc_close(pj)
            dist.barrier(group=self.group)
            if own.value:
                C.lib().tops_gla_p2p_free(own)
            raise RuntimeError(f"peer-memory regions could not be set up: rank {failed[0][0]}: {failed[0][1]}")
        table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        dist.barrier(group=self.group)  # every region is mapped everywhere before the first push
        reg = self.regions[shape] = (own, mapped, table)
        return reg

    def prepare(self, shape) -> None:
        """Set up the regions for states of ``shape`` = (N, H, K, V) now (collective).  Raises
        RuntimeError on every rank if any rank could not allocate or map them."""
        self._region(tuple(int(x) for x in shape))

    def check_peers(self) -> None:
        """Raise PeerLostError if a peer is gone (before any exchange kernel is launched)."""
        if self.watchdog is not None:
            self.watchdog.check()

    def abort(self) -> None:
        """Stop watching the peers (there is no communicator; the kernels' own waits are
        bounded)."""
        if self.watchdog is not None:
            self.watchdog.close()
            self.watchdog = None

    def wait(self, timeout_s: float, stream=None) -> None:
        """Wait on the host, at most ``timeout_s``, for the exchanges enqueued so far; raise
        TopsError at the deadline or if a device-side wait for a peer gave up."""
        ev = torch.cuda.Event()
        ev.record(stream if stream is not None else torch.cuda.current_stream(self.device))
        deadline = time.monotonic() + timeout_s
        while not ev.query():
            if time.monotonic() > deadline:
                raise self._C.TopsError("P2PStateExchange.wait", -5, f"exchange not done after {timeout_s} s")
            time.sleep(0.0002)
        code = int(self._C.lib().tops_gla_device_error())
        if code:
            raise self._C.TopsError("P2PStateExchange.wait", -5, f"device wait for a peer gave up (error {code})")

    def _run(self, backward: bool, local: torch.Tensor, decay: torch.Tensor, boundary, want_total: bool):
        C = self._C
        self.check_peers()
        local = local.float().contiguous()
        decay = decay.float().contiguous()
        boundary = None if boundary is None else boundary.float().contiguous()
        shape = tuple(local.shape)
        own, _, table = self._region(shape)
        out = torch.empty_like(local)
        total = torch.empty_like(local) if want_total else None
        a = self._args(shape, backward)
        a.local_state, a.decay, a.boundary = C.ptr(local), C.ptr(decay), C.ptr(boundary)
        a.out, a.total, a.regions, a.own_region = C.ptr(out), C.ptr(total), C.ptr(table), own.value
        C.call("tops_gla_p2p_exchange", a, C.stream_of(local))
        return out, total

    def forward(self, S, D, h0=None):
        """-> (this rank's incoming state, the whole sequence's final state)."""
        return self._run(False, S, D, h0, True)

    def backward(self, L, D, dht=None):
        """-> the final-state gradient this rank's backward must use."""
        return self._run(True, L, D, dht, False)[0]

    def push_args(self, shape):
        """The ``_C.P2PArgs`` naming this group's regions for states of ``shape`` (N, H, K, V),
        for a kernel that pushes this rank's state itself (the span-begin entry points);
        checks the peers first."""
        self.check_peers()
        shape = tuple(int(x) for x in shape)
        own, _, table = self._region(shape)
        a = self._args(shape)
        a.regions, a.own_region = self._C.ptr(table), own.value
        return a

    def combine(self, backward: bool, shape, boundary=None, want_total: bool = False, device=None):
        """The receiving half after a fused push: wait for every rank's push of this epoch and
        fold the prefix (forward: -> (incoming state, final state)) or suffix (backward: ->
        (final-state gradient, None))."""
        C = self._C
        shape = tuple(int(x) for x in shape)
        own, _, table = self._region(shape)
        dev = self.device if device is None else device
        boundary = None if boundary is None else boundary.float().contiguous()
        out = torch.empty(shape, dtype=torch.float32, device=dev)
        total = torch.empty(shape, dtype=torch.float32, device=dev) if want_total else None
        a = self._args(shape, backward)
        a.boundary, a.out, a.total = C.ptr(boundary), C.ptr(out), C.ptr(total)
        a.regions, a.own_region = C.ptr(table), own.value
        C.call("tops_gla_p2p_combine", a, C.stream_of(out))
        return out, total

    def close(self):
        """Unmap and free the regions (collective: no rank frees its region while another may
        still write into it)."""
        if self.regions:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for own, mapped, _ in self.regions.values():
                for p in mapped:
                    self._C.call("tops_gla_ipc_close", p)
            dist.barrier(group=self.group)
            for own, _, _ in self.regions.values():
                self._C.call("tops_gla_p2p_free", own)
            self.regions = {}
        if self.watchdog is not None:
            self.watchdog.close()
            self.watchdog = None


def shard(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """Contiguous slice ``rank`` of ``world`` along ``dim`` (batch or heads); sizes must divide."""
    n = x.shape[dim]
    assert n % world == 0, f"dimension {dim} of size {n} does not split over {world} ranks"
    s = n // world
    return x.narrow(dim, rank * s, s)


def all_gather_stack(x: torch.Tensor, group=None) -> torch.Tensor:
    """[world, *x.shape] stack of every rank's ``x`` (one all-gather)."""
    world = dist.get_world_size(group)
    out = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(out, x.contiguous(), group=group)
    return torch.stack(out, 0)


def prefix_states(S: torch.Tensor, D: torch.Tensor, h0: torch.Tensor | None) -> torch.Tensor:
    """Incoming states of every rank: H_0 = h0 (or 0), H_{r+1} = D_r * H_r + S_r.

    S: [R, N, H, K, V] span final states from a zero state; D: [R, N, H, K] span decays.
    Returns [R, N, H, K, V].
    """
    R = S.shape[0]
    H = torch.zeros_like(S[0]) if h0 is None else h0.to(S.dtype).clone()
    out = []
    for r in range(R):
        out.append(H)
        H = D[r][..., None] * H + S[r]
    return torch.stack(out, 0)


def suffix_grads(dh0_local: torch.Tensor, D: torch.Tensor, dht: torch.Tensor | None) -> torch.Tensor:
    """Gradient w.r.t. every rank's final state: G_{R-1} = dht (or 0), G_{r-1} = D_r * G_r + dh0_local_r.

    dh0_local: [R, N, H, K, V] gradient of each span's own loss w.r.t. its incoming state
    (computed with a zero final-state gradient); D: [R, N, H, K].  Returns [R, N, H, K, V]
    where entry r is the final-state gradient rank r must use in its backward.
    """
    R = dh0_local.shape[0]
    G = torch.zeros_like(dh0_local[0]) if dht is None else dht.to(dh0_local.dtype).clone()
    out = [None] * R
    for r in range(R - 1, -1, -1):
        out[r] = G
        G = D[r][..., None] * G + dh0_local[r]
    return torch.stack(out, 0)


def _exchange_forward(S, D, h0, group, exchange):
    """(this rank's incoming state, the whole sequence's final state) from every rank's (S, D)."""
    if exchange is not None:
        return exchange.forward(S, D, h0)
    rank = dist.get_rank(group)
    S_all = all_gather_stack(S, group)
    D_all = all_gather_stack(D.to(S.dtype), group)
    H_all = prefix_states(S_all, D_all, h0)
    return H_all[rank], D_all[-1][..., None] * H_all[-1] + S_all[-1]


def _exchange_backward(L, D, dht, group, exchange):
    """The final-state gradient this rank's backward must use, from every rank's (L, D)."""
    if exchange is not None:
        return exchange.backward(L, D, dht)
    L_all = all_gather_stack(L, group)
    D_all = all_gather_stack(D.to(L.dtype), group)
    return suffix_grads(L_all, D_all, dht)[dist.get_rank(group)]


def seq_parallel_forward_phased(begin: Callable, finish: Callable, h0=None, group=None,
                                exchange: NcclStateExchange | None = None):
    """Forward of one rank's span in two phases (no recomputation).

    begin() -> (S, D): everything that does not depend on the incoming state, returning the
    span's final state from a zero state and its decay; finish(H_in) -> o completes the span
    from its incoming state.  Returns (o, H_in, ht_global, D).
    """
    S, D = begin()
    H_in, ht_global = _exchange_forward(S, D, h0, group, exchange)
    return finish(H_in), H_in, ht_global, D


def seq_parallel_backward_phased(begin: Callable, finish: Callable, D: torch.Tensor, dht=None, group=None,
                                 exchange: NcclStateExchange | None = None):
    """Backward of one rank's span in two phases: begin() -> the gradient of the span's own loss
    w.r.t. its incoming state; finish(G) -> the gradients, G being the final-state gradient from
    the later spans (``dht`` for the last)."""
    return finish(_exchange_backward(begin(), D, dht, group, exchange))


def seq_parallel_forward(local_fwd: Callable, span_decay: Callable, q, k, v, g, h0=None, group=None,
                         local_final: Callable | None = None, exchange: NcclStateExchange | None = None):
    """Forward of one rank's span.

    local_fwd(q, k, v, g, h0) -> (o, final_state) runs the chunked forward on this span;
    span_decay(g) -> D [N, H, K] is exp of the span's gate sums; local_final(q, k, v, g)
    -> the span's final state from a zero state (default: local_fwd's).  ``h0`` (rank 0's
    initial state) is read on every rank (pass the same tensor or None).  ``exchange``: use the
    C ABI's NCCL exchange instead of torch all-gathers.  Returns (o, H_in, ht_global) where
    H_in is this rank's incoming state and ht_global the final state of the whole sequence
    (identical on all ranks).
    """
    S = local_final(q, k, v, g) if local_final is not None else local_fwd(q, k, v, g, None)[1]
    D = span_decay(g)
    H_in, ht_global = _exchange_forward(S, D, h0, group, exchange)
    o, _ = local_fwd(q, k, v, g, H_in)
    return o, H_in, ht_global


def seq_parallel_backward(local_bwd: Callable, D: torch.Tensor, H_in, do, dht=None, group=None,
                          local_dh0: Callable | None = None, exchange: NcclStateExchange | None = None):
    """Backward of one rank's span.

    local_bwd(H_in, do, dht) -> (dq, dk, dv, dg, dh0) runs the chunked backward of this span
    from its incoming state; local_dh0(H_in, do) -> dh0 of the span's own loss alone
    (default: local_bwd's).  D: this span's decay [N, H, K].  ``dht`` is the gradient of the
    whole sequence's final state (read by the last rank).  Returns (dq, dk, dv, dg, dh0) where
    dh0 is the gradient w.r.t. this rank's incoming state (rank 0: the user's initial state).
    """
    dh0_local = local_dh0(H_in, do) if local_dh0 is not None else local_bwd(H_in, do, None)[-1]
    return local_bwd(H_in, do, _exchange_backward(dh0_local, D, dht, group, exchange))


class _SeqParallelChunkGLA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, h0, scale, chunk_size, group, exchange):
        from .ops.gla import _core

        p = _core.make_plan(q, v.shape[-1], chunk_size, None, scale)
        ctx.plan, ctx.group, ctx.has_h0, ctx.exchange = p, group, h0 is not None, exchange
        if _core.span_saved_size(p, g) > 0 and getattr(exchange, "fused_push", False):
            # tensor-core path, state pushed to the peers by the kernel that computes it
            shape = (p.N, p.H, p.K, p.V)
            D, blk = _core.fwd_span_begin_p2p(p, q, k, v, g, exchange.push_args(shape))
            H_in, ht = exchange.combine(False, shape, h0, True, q.device)
            o = _core.fwd_span_finish(p, q, k, v, g, H_in, blk)[0]
            ctx.save_for_backward(q, k, v, g, H_in, D)
            ctx.phased, ctx.fwd_saved = True, blk
            return o, ht
        if _core.span_saved_size(p, g) > 0:
            # tensor-core path: two phases, nothing computed twice
            blk = {}

            def begin():
                S, D, blk["b"] = _core.fwd_span_begin(p, q, k, v, g)
                return S, D

            def finish(h_in):
                return _core.fwd_span_finish(p, q, k, v, g, h_in, blk["b"])[0]

            o, H_in, ht, D = seq_parallel_forward_phased(begin, finish, h0, group, exchange)
            ctx.save_for_backward(q, k, v, g, H_in, D)
            ctx.phased, ctx.fwd_saved = True, blk["b"]
            return o, ht
        saved = {}

        def local_fwd(q_, k_, v_, g_, h_):
            o, ht, sv = _core.chunk_fwd(p, q_, k_, v_, g_, h_, True, save=True)
            saved.update(sv)
            return o, ht

        def local_final(q_, k_, v_, g_):  # state scan only
            return _core.final_state(p, q_, k_, v_, g_, None)

        o, H_in, ht = seq_parallel_forward(local_fwd, lambda g_: _core.span_decay(p, g_), q, k, v, g, h0, group,
                                           local_final=local_final, exchange=exchange)
        ctx.save_for_backward(q, k, v, g, H_in, None)
        ctx.phased, ctx.fwd_saved = False, saved
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        from .ops.gla import _core

        q, k, v, g, H_in, D = ctx.saved_tensors
        p, sv = ctx.plan, ctx.fwd_saved
        rank = dist.get_rank(ctx.group)
        want = ctx.has_h0 and rank == 0
        do = do.contiguous().to(q.dtype)
        dht = None if dht is None else dht.float()
        if ctx.phased and getattr(ctx.exchange, "fused_push", False):
            shape = (p.N, p.H, p.K, p.V)
            ws = _core.bwd_span_begin_p2p(p, q, k, v, g, do, sv, D, ctx.exchange.push_args(shape))
            G = ctx.exchange.combine(True, shape, dht, False, q.device)[0]
            dq, dk, dv, dg, dh0 = _core.bwd_span_finish(p, q, k, v, g, do, G, sv, ws, want_dh0=want)
            return dq, dk, dv, dg, dh0, None, None, None, None
        if ctx.phased:
            ws = {}

            def begin():
                L, ws["w"] = _core.bwd_span_begin(p, q, k, v, g, do, sv)
                return L

            def finish(G):
                return _core.bwd_span_finish(p, q, k, v, g, do, G, sv, ws["w"], want_dh0=want)

            dq, dk, dv, dg, dh0 = seq_parallel_backward_phased(begin, finish, D, dht, ctx.group, ctx.exchange)
            return dq, dk, dv, dg, dh0, None, None, None, None

        def local_bwd(h_in, do_, dht_):
            return _core.chunk_bwd(p, q, k, v, g, h_in, do_, dht_, sv.get("g_cumsum"), sv.get("A"), sv.get("h"),
                                   want_dh0=True, block=sv.get("block"))

        def local_dh0(h_in, do_):  # reverse state scan only
            return _core.initial_state_grad(p, q, k, v, g, h_in, do_, None, block=sv.get("block"))

        D = _core.span_decay(p, g)
        dq, dk, dv, dg, dh0 = seq_parallel_backward(local_bwd, D, H_in, do, dht, ctx.group,
                                                    local_dh0=local_dh0, exchange=ctx.exchange)
        return dq, dk, dv, dg, dh0 if want else None, None, None, None, None


def chunk_gla_seq_parallel(q, k, v, g, scale=None, initial_state=None, chunk_size=64, group=None, exchange=None):
    """chunk_gla over a sequence split into contiguous spans, one per rank (differentiable).

    q, k, g: this rank's span [B, T_r, H, K]; v: [B, T_r, H, V] (CUDA tensors, same T_r on
    every rank).  initial_state: [B, H, K, V] state before rank 0's span (or None).
    Returns (o of this span, final state of the whole sequence).  The only communication
    is two all-gathers of [B, H, K, V] fp32 states (+ [B, H, K] decays) per direction
    (torch.distributed, or the C ABI's NCCL exchange when ``exchange`` is an
    ``NcclStateExchange``).  On the tensor-core path the span runs in two phases (the C
    ABI's tops_gla_chunk_{fwd,bwd}_span_{begin,finish}): the work that does not depend on
    the incoming state runs before the exchange and is not repeated after it.
    """
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return _SeqParallelChunkGLA.apply(q, k, v, g.float().contiguous(), initial_state, float(scale), int(chunk_size),
                                      group, exchange)
