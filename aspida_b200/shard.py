"""Multi-GPU partitioning of the attention path (one process per GPU).

The reference has no multi-GPU inference (its only distributed code is a TCP
gradient exchange for training, gpu/dp_node.cu), so these are new parts:

* Batched decode and prefill shard by sequence: independent units, no
  collective on the data path. ``plan_sequences`` balances the KV bytes
  (sum of lengths) over ranks with a longest-first greedy assignment.
* Single long-sequence decode splits the KV cache into contiguous chunks
  (``kv_chunks``); each rank attends its chunk and produces the split-KV
  partial (m, l, o) per query head (aspida_attn_decode_partial), the ranks
  exchange the partials and every rank merges them with the log-sum-exp
  merge of gpu/fattn_sk.cu:84-97. The payload is nq*(hd+2) floats per
  sequence per rank (33 KB at 64 heads x hd 128), so the exchange is
  latency-bound. Two transports:
    - "p2p" (default): one kernel stores this rank's partial into every
      rank's receive buffer over NVLink (buffers shared once through CUDA IPC
      handles, :class:`PeerExchange`), waits for all ranks' partials of the
      step and merges (aspida_attn_exchange_merge);
    - "nccl": an all-gather of the packed partials, then
      aspida_attn_merge_strided.

Failures: a collective that fails (a rank died or timed out) raises
:class:`ShardError`; no rank waits forever, the process-group timeout bounds
every exchange.
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence, Tuple

import torch


class ShardError(RuntimeError):
    pass


def plan_sequences(lens: Sequence[int], world: int) -> List[List[int]]:
    """Assign sequence indices to ranks, balancing sum(len) (longest first)."""
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    out: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    for r in out:
        r.sort()
    return out


def kv_chunks(length: int, world: int, align: int = 16) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) key ranges of a cache of `length` rows, one per
    rank, as equal as possible with boundaries on `align`-row multiples."""
    if world <= 0:
        raise ValueError("world must be positive")
    units = (length + align - 1) // align
    out = []
    for r in range(world):
        lo = min(length, (r * units // world) * align)
        hi = min(length, ((r + 1) * units // world) * align)
        out.append((lo, hi))
    return out


def pack_partials(m: torch.Tensor, l: torch.Tensor, o: torch.Tensor) -> torch.Tensor:
    """(m [B,nq], l [B,nq], o [B,nq,hd]) -> one flat f32 buffer for the exchange."""
    return torch.cat([m.reshape(-1), l.reshape(-1), o.reshape(-1)])


def unpack_partials(buf: torch.Tensor, world: int, B: int, nq: int, hd: int):
    """Gathered [world * per] buffer -> m, l [world, B*nq]; o [world, B*nq, hd]."""
    per = B * nq * (hd + 2)
    g = buf.reshape(world, per)
    m = g[:, :B * nq]
    l = g[:, B * nq:2 * B * nq]
    o = g[:, 2 * B * nq:].reshape(world, B * nq, hd)
    return m.contiguous(), l.contiguous(), o.contiguous()


def exchange_partials(m, l, o, group=None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """All-gather every rank's partial (one collective)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    B, nq = m.shape
    hd = o.shape[-1]
    mine = pack_partials(m, l, o)
    gathered = torch.empty(world * mine.numel(), dtype=mine.dtype, device=mine.device)
    try:
        dist.all_gather_into_tensor(gathered, mine, group=group)
    except Exception as e:  # a peer died, timed out or the group was torn down
        raise ShardError(f"partial exchange failed: {e}") from e
    return unpack_partials(gathered, world, B, nq, hd)


class PeerExchange:
    """Per-rank NVLink receive buffers for the fused exchange + merge.

    Each rank allocates its buffer in the library (zero-filled) and shares its
    CUDA IPC handle with the group once; every rank then maps every other
    rank's buffer. ``__call__`` runs one step: all ranks must call it once per
    step, in the same order (the step number tags the arrivals)."""

    def __init__(self, rows: int, hd: int, group=None, wait_limit: int = 0):
        import ctypes as C
        import torch.distributed as dist
        from . import _lib
        from .attention import GPUError
        self._C, self._lib, self.group = C, _lib.load(), group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer exchange supports up to 8 ranks")
        self.rows, self.hd, self.step = rows, hd, 0
        # The kernel sets this pinned (device-visible) word when its wait for a
        # peer runs out; the host reads it without synchronising the stream.
        # After a timeout the two-bank reuse guarantee no longer holds, so the
        # exchange refuses every further step.
        self.wait_limit = int(wait_limit)
        self.fail_word = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.failed = False
        # every rank takes part in the same collectives whatever fails
        # locally, so a failure is seen by all ranks and none is left waiting
        nbytes = self._lib.aspida_attn_peer_buffer_size(self.world, rows, hd)
        own = C.c_void_p()
        handle = (C.c_char * 64)()
        rc = self._lib.aspida_attn_peer_alloc(nbytes, C.byref(own), handle)
        self._own = own.value if rc == 0 else None
        self._mapped = []
        handles = [None] * self.world
        try:
            dist.all_gather_object(handles, bytes(handle) if rc == 0 else None, group=group)
        except Exception as e:
            self.close(barrier=False)
            raise ShardError(f"peer handle exchange failed: {e}") from e
        if any(h is None for h in handles):
            self.close(barrier=False)
            raise ShardError("peer buffer allocation failed on a rank")
        ptrs, ok = [], True
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = C.c_void_p()
            if ok and self._lib.aspida_attn_peer_open((C.c_char * 64).from_buffer_copy(h),
                                                      C.byref(p)) == 0:
                self._mapped.append(p.value)
                ptrs.append(p.value)
            else:
                ok = False
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=torch.device(
            "cuda", torch.cuda.current_device()))
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
        if int(flag.item()) != 0:
            self.close(barrier=False)
            raise ShardError("peer buffer mapping failed on a rank (no peer access?)")
        self.table = (C.c_void_p * self.world)(*ptrs)

    def __call__(self, part: torch.Tensor, out: torch.Tensor, gate: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
        from .attention import GPUError, _stream
        self._raise_if_failed()
        self.step += 1
        rc = self._lib.aspida_attn_exchange_merge_ex(
            part.data_ptr(), self.table, self.world, self.rank, self.step,
            None if gate is None else gate.data_ptr(), out.data_ptr(), self.rows, self.hd,
            self.fail_word.data_ptr(), self.wait_limit, _stream(stream))
        if rc:
            raise GPUError(rc, "exchange_merge")
        return out

    def _raise_if_failed(self):
        if self.failed or int(self.fail_word[0]) != 0:
            self.failed = True
            raise ShardError(f"peer exchange timed out waiting for a rank (step {self.step}); "
                             "its buffers are no longer usable")

    def check(self, stream=None):
        """Wait for the last step on ``stream`` and raise :class:`ShardError`
        if any exchange so far gave up waiting for a peer. Without this call
        a timeout is raised at the start of the next step."""
        (stream or torch.cuda.current_stream()).synchronize()
        self._raise_if_failed()

    def close(self, barrier: bool = True):
        """Unmap the peers' buffers and free this rank's (after a barrier, so
        no rank still stores into it)."""
        import torch.distributed as dist
        torch.cuda.synchronize()
        if barrier:
            try:
                dist.barrier(group=self.group)
            except Exception:
                pass
        for p in getattr(self, "_mapped", []):
            self._lib.aspida_attn_peer_close(p)
        self._mapped = []
        if getattr(self, "_own", None) is not None:
            self._lib.aspida_attn_peer_free(self._own)
            self._own = None


class SeqParallelDecode:
    """Sequence-parallel decode with every buffer allocated once.

    Per call: the split-KV partial kernel writes this rank's (m, l, o) straight
    into a packed send buffer [m | l | o]; then, with transport "p2p", one
    kernel exchanges it over NVLink and merges (:class:`PeerExchange`); with
    "nccl", one all-gather fills the receive buffer [world][m | l | o] and the
    strided merge kernel reads it in place. No host synchronisation and no
    extra device copies. ``close()`` releases the peer buffers.

    K_chunks / V_chunks: this rank's fp16 chunk [rows >= n_local, nkv*hd] of
    each of the B sequences' caches; rows 0..n_local-1 are attended."""

    def __init__(self, K_chunks, V_chunks, n_local: int, nq: int, nkv: int, hd: int, *,
                 scale: Optional[float] = None, softcap: float = 0.0, group=None,
                 transport: str = "p2p"):
        import math
        import torch.distributed as dist
        from . import attention as ab
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.B = len(K_chunks)
        self.nq, self.nkv, self.hd, self.n = nq, nkv, hd, n_local
        self.scale = 1.0 / math.sqrt(hd) if scale is None else scale
        self.softcap = softcap
        dev = K_chunks[0].device
        self.rows = self.B * nq
        self.per = self.rows * (hd + 2)
        self.send = torch.empty(self.per, dtype=torch.float32, device=dev)
        self.recv = torch.empty(self.world * self.per, dtype=torch.float32, device=dev)
        self.out = torch.empty(self.B, nq * hd, dtype=torch.float32, device=dev)
        self.Kt, self.Vt = ab.ptr_table(list(K_chunks), dev), ab.ptr_table(list(V_chunks), dev)
        self.lo = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.hi = torch.full((self.B,), n_local, dtype=torch.int32, device=dev)
        nbytes = ab.decode_workspace_size(self.B, nq, nkv, hd, max(1, n_local))
        self.ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        self.pos = torch.full((self.B,), n_local - 1, dtype=torch.int32, device=dev)
        if transport not in ("p2p", "nccl"):
            raise ValueError("transport must be 'p2p' or 'nccl'")
        self.transport = transport if self.world > 1 else "local"
        self.px = PeerExchange(self.rows, hd, group) if self.transport == "p2p" else None

    def close(self):
        if self.px is not None:
            self.px.close()
            self.px = None

    def check(self, stream=None):
        """Raise :class:`ShardError` if an exchange so far timed out (p2p
        transport; waits for the stream first)."""
        if self.px is not None:
            self.px.check(stream)

    def __call__(self, q: torch.Tensor, gate: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
        from . import _lib
        from .attention import GPUError, _stream
        lib = _lib.load()
        st = _stream(stream)
        if self.world == 1:
            # one rank holds the whole range: plain decode, no partial round trip
            rc = lib.aspida_attn_decode(
                q.data_ptr(), None if gate is None else gate.data_ptr(), self.Kt.data_ptr(),
                self.Vt.data_ptr(), self.pos.data_ptr(), None, self.out.data_ptr(), self.B,
                self.nq, self.nkv, self.hd, self.scale, 0, self.softcap, max(1, self.n), 0,
                self.ws.data_ptr(), self.ws.numel(), st)
            if rc:
                raise GPUError(rc, "decode")
            return self.out
        sp = self.send.data_ptr()
        rc = lib.aspida_attn_decode_partial(
            q.data_ptr(), self.Kt.data_ptr(), self.Vt.data_ptr(), self.lo.data_ptr(),
            self.hi.data_ptr(), sp, sp + 4 * self.rows, sp + 8 * self.rows, self.B, self.nq,
            self.nkv, self.hd, self.scale, self.softcap, max(1, self.n), 0, self.ws.data_ptr(),
            self.ws.numel(), st)
        if rc:
            raise GPUError(rc, "decode_partial")
        if self.transport == "p2p":
            return self.px(self.send, self.out, gate=gate, stream=stream)
        src = self.send
        if self.world > 1:
            import torch.distributed as dist
            try:
                dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
            except Exception as e:  # a peer died, timed out or the group was torn down
                raise ShardError(f"partial exchange failed: {e}") from e
            src = self.recv
        rp = src.data_ptr()
        rc = lib.aspida_attn_merge_strided(
            rp, rp + 4 * self.rows, rp + 8 * self.rows, None if gate is None else gate.data_ptr(),
            self.out.data_ptr(), self.world, self.rows, self.hd, self.per, st)
        if rc:
            raise GPUError(rc, "merge_strided")
        return self.out


def seq_parallel_decode(q: torch.Tensor, K_local, V_local, n_local: int, nq: int, nkv: int,
                        hd: int, *, gate: Optional[torch.Tensor] = None,
                        scale: Optional[float] = None, softcap: float = 0.0,
                        group=None, transport: str = "p2p") -> torch.Tensor:
    """One-shot form of :class:`SeqParallelDecode`. q [B, nq*hd] f32 (identical
    on every rank); K_local / V_local: one tensor when B = 1, else a sequence
    of B chunks. Returns the merged [B, nq*hd] output on every rank."""
    Ks = [K_local] if isinstance(K_local, torch.Tensor) else list(K_local)
    Vs = [V_local] if isinstance(V_local, torch.Tensor) else list(V_local)
    if len(Ks) != q.shape[0] or len(Vs) != q.shape[0]:
        raise ValueError("one K/V chunk per sequence")
    op = SeqParallelDecode(Ks, Vs, n_local, nq, nkv, hd, scale=scale, softcap=softcap,
                           group=group, transport=transport)
    try:
        return op(q, gate=gate).clone()
    finally:
        op.close()
