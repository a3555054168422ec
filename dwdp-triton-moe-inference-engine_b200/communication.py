"""Python surface of the DWDP communication engine, with the names of the
reference's pybind module (DWDP/communication/bindings.cpp:32-111):
``export_ipc_handle``, ``CommunicationEngine``, ``PeerTopology``,
``TransferScheduler``, ``TransferState``, ``CommunicationPath`` and
``CommunicationPolicy``. All of them call the C ABI (include/dwdp_b200.h)."""
from __future__ import annotations

import ctypes
import enum

import torch

from . import _lib


class TransferState(enum.IntEnum):
    CREATED = 0
    QUEUED = 1
    RUNNING = 2
    WAITING = 3
    COMPLETED = 4
    FAILED = 5
    CANCELLED = 6


class CommunicationPath(enum.IntEnum):
    LOCAL = 0
    P2P = 1
    IPC = 2
    COPY = 3


class ResidentState(enum.IntEnum):
    NONE = 0
    STAGED = 1
    ACTIVE = 2


def _chk(rc: int, what: str) -> None:
    _lib.check(rc, what, engine=True)


def export_ipc_handle(tensor_or_ptr) -> bytes:
    """IPC handle of the allocation holding the pointer, followed by the pointer's
    8-byte little-endian offset inside that allocation (so the importer can reach
    a sub-allocated tensor)."""
    ptr = tensor_or_ptr.data_ptr() if isinstance(tensor_or_ptr, torch.Tensor) else int(tensor_or_ptr)
    lib = _lib.load()
    n = int(lib.dwdp_ipc_handle_bytes())
    buf = ctypes.create_string_buffer(n)
    off = ctypes.c_size_t(0)
    _chk(lib.dwdp_export_ipc_handle(ptr, buf, ctypes.byref(off)), "export_ipc_handle")
    return buf.raw + int(off.value).to_bytes(8, "little")


def split_ipc_handle(blob: bytes) -> tuple[bytes, int]:
    n = int(_lib.load().dwdp_ipc_handle_bytes())
    if len(blob) != n + 8:
        raise ValueError(f"IPC blob must be {n + 8} bytes, got {len(blob)}")
    return blob[:n], int.from_bytes(blob[n:], "little")


class PeerTopology:
    """Peer-access queries (topology.cpp:17-41), cached per pair."""

    def __init__(self) -> None:
        self._cache: dict[tuple[int, int], bool] = {}

    def can_access(self, src: int, dst: int) -> bool:
        key = (src, dst)
        if key not in self._cache:
            out = ctypes.c_int(0)
            _chk(_lib.load().dwdp_peer_can_access(src, dst, ctypes.byref(out)), "peer_can_access")
            self._cache[key] = bool(out.value)
        return self._cache[key]

    canAccess = can_access


class CommunicationPolicy:
    """Path selection (communication_policy.cpp:5-17)."""

    def __init__(self, local_gpu: int) -> None:
        self.local_gpu = local_gpu

    def decide(self, *, owner_gpu: int, resident: ResidentState = ResidentState.NONE,
               has_ipc_handle: bool = False, peer_access: bool = False) -> CommunicationPath:
        return CommunicationPath(_lib.load().dwdp_policy_decide(
            self.local_gpu, owner_gpu, int(resident), int(has_ipc_handle), int(peer_access)))


class TransferScheduler:
    """Priority queue of expert transfers with coalescing, two retries, cancel
    while queued and a bounded take (transfer_scheduler.cpp:15-104)."""

    def __init__(self) -> None:
        h = ctypes.c_void_p()
        _chk(_lib.load().dwdp_sched_create(ctypes.byref(h)), "sched_create")
        self._h = h

    def submit(self, expert_id: int, priority: int = 0) -> None:
        rc = _lib.load().dwdp_sched_submit(self._h, expert_id, priority)
        if rc == _lib.DWDP_ERR_INVALID_ARGUMENT:
            raise ValueError(_lib.engine_last_error())
        if rc == _lib.DWDP_ERR_STATE:
            raise RuntimeError(_lib.engine_last_error())
        _chk(rc, "submit")

    def take(self, timeout_ms: int = 1000) -> int | None:
        """Next expert id (now RUNNING); None once closed and drained."""
        out = ctypes.c_int(-1)
        _chk(_lib.load().dwdp_sched_take(self._h, timeout_ms, ctypes.byref(out)), "take")
        return None if out.value < 0 else out.value

    def complete(self, expert_id: int) -> None:
        _chk(_lib.load().dwdp_sched_complete(self._h, expert_id), "complete")

    def fail(self, expert_id: int, retryable: bool) -> None:
        _chk(_lib.load().dwdp_sched_fail(self._h, expert_id, int(retryable)), "fail")

    def cancel(self, expert_id: int) -> None:
        _chk(_lib.load().dwdp_sched_cancel(self._h, expert_id), "cancel")

    def close(self) -> None:
        _chk(_lib.load().dwdp_sched_close(self._h), "close")

    def state(self, expert_id: int) -> tuple[TransferState, int]:
        st, rt = ctypes.c_int(0), ctypes.c_int(0)
        _chk(_lib.load().dwdp_sched_state(self._h, expert_id, ctypes.byref(st), ctypes.byref(rt)), "state")
        return TransferState(st.value), rt.value

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        try:
            if h is not None and h.value:
                _lib.load().dwdp_sched_destroy(h)
        except Exception:  # noqa: BLE001 - interpreter teardown
            pass
        self._h = None


class CommunicationEngine:
    """Expert-slab prefetch engine (communication_engine.cpp; bindings.cpp:39-60).

    Two ways to drive it:

    * the reference's surface (``CommunicationEngine(device_id)``, bindings.cpp:39-60):
      ``initialize(staging_bytes)``, ``register_expert(id, ptr, size)`` /
      ``register_ipc_expert(id, handle, size)``, ``prefetch(id)`` (copy a remote expert
      into the NEXT staging buffer), ``wait(id)`` (order the current stream after that
      copy), ``swap_buffers()`` (the next buffer becomes current, after the compute that
      read the current one was queued), ``is_resident(id)``, ``get_resident_pointer(id)``,
      ``get_weight(id)``, ``release(id)``, ``initialized()``, ``shutdown()``. Staging is
      two buffers with one fixed slot of ``staging_bytes`` per registered remote expert,
      created on the first prefetch (the reference's buffers hold one expert at a time);
    * whole layers at once, as the DWDP path uses it: ``initialize(slot_bytes, num_slots,
      num_buffers)``, ``prefetch_into(ids, buffer)`` copies every listed remote expert
      into ``buffer`` on the engine's greatest-priority copy streams, ``wait_buffer(buffer)``
      orders the current torch stream after those copies."""

    def __init__(self, device_id: int = 0) -> None:
        self.device_id = device_id
        self._h = None
        self._pending: list[tuple] | None = None  # registrations made before a deferred create
        self._slot_bytes = 0
        self.num_buffers = 0
        self._current = 0
        self._where: dict[int, int] = {}  # remote expert -> staging buffer of its last prefetch
        self._local: set[int] = set()

    def initialize(self, staging_bytes: int, num_slots: int | None = None, num_buffers: int = 2) -> None:
        if self.initialized():
            raise RuntimeError("engine already initialized")
        if num_slots is None:  # the reference's form: staging created once the experts are known
            if staging_bytes <= 0:
                raise ValueError("staging_bytes must be > 0")
            self._pending = []
            self._slot_bytes = int(staging_bytes)
            self.num_buffers = 2
            return
        h = ctypes.c_void_p()
        self._slot_bytes = int(staging_bytes)
        _chk(_lib.load().dwdp_engine_create(self.device_id, self._slot_bytes, num_slots, num_buffers,
                                            ctypes.byref(h)), "engine_create")
        self._h = h
        self.num_buffers = num_buffers

    def initialized(self) -> bool:
        return self._h is not None or self._pending is not None

    def _eng(self):
        if self._pending is not None:  # first use of a reference-form engine: create, replay
            pending, self._pending = self._pending, None
            n_remote = sum(1 for p in pending if p[0] != "local")
            h = ctypes.c_void_p()
            _chk(_lib.load().dwdp_engine_create(self.device_id, self._slot_bytes, max(1, n_remote), 2,
                                                ctypes.byref(h)), "engine_create")
            self._h = h
            for kind, *args in pending:
                getattr(self, "_register_" + kind)(*args)
        if self._h is None:
            raise RuntimeError("communication engine is not initialized")
        return self._h

    def _register_local(self, expert_id: int, ptr: int, size_bytes: int) -> None:
        _chk(_lib.load().dwdp_engine_register_local(self._h, expert_id, ptr, size_bytes), "register_expert")
        self._local.add(expert_id)

    def _register_ipc(self, expert_id: int, handle: bytes, off: int, size_bytes: int, owner_device: int) -> None:
        _chk(_lib.load().dwdp_engine_register_ipc(self._h, expert_id, handle, off, size_bytes, owner_device),
             "register_ipc_expert")
        self._local.discard(expert_id)

    def _register_peer(self, expert_id: int, ptr: int, size_bytes: int, owner_device: int) -> None:
        _chk(_lib.load().dwdp_engine_register_peer(self._h, expert_id, ptr, size_bytes, owner_device),
             "register_peer_expert")
        self._local.discard(expert_id)

    def _register(self, kind: str, *args) -> None:
        if self._pending is not None:
            if kind != "local" and args[-2] > self._slot_bytes:  # (..., size_bytes, owner_device)
                raise ValueError("expert exceeds the staging capacity")
            self._pending.append((kind, *args))
            if kind == "local":
                self._local.add(args[0])
            return
        self._eng()
        getattr(self, "_register_" + kind)(*args)

    def register_expert(self, expert_id: int, ptr: int, size_bytes: int) -> None:
        """A local expert (the reference's register_expert): used in place, never copied."""
        self._register("local", expert_id, int(ptr), int(size_bytes))

    def register_ipc_expert(self, expert_id: int, handle_blob: bytes, size_bytes: int, owner_device: int = -1,
                            extra_offset: int = 0) -> None:
        handle, off = split_ipc_handle(handle_blob)
        self._register("ipc", expert_id, handle, off + extra_offset, int(size_bytes), owner_device)

    def register_peer_expert(self, expert_id: int, ptr: int, size_bytes: int, owner_device: int) -> None:
        self._register("peer", expert_id, int(ptr), int(size_bytes), owner_device)

    # ------------------------------------------------------------------ whole-layer form
    def prefetch_into(self, expert_ids, buffer: int = 0, after_current_stream: bool = True) -> None:
        ids = [int(expert_ids)] if isinstance(expert_ids, int) else [int(e) for e in expert_ids]
        arr = (ctypes.c_int * max(1, len(ids)))(*ids)
        after = torch.cuda.current_stream(self.device_id).cuda_stream if after_current_stream else None
        _chk(_lib.load().dwdp_engine_prefetch(self._eng(), arr, len(ids), buffer, after), "prefetch")
        for e in ids:
            if e not in self._local:
                self._where[e] = buffer

    def issue_order(self, plan) -> list:
        """The plan's descriptors in the order the TransferScheduler releases their experts
        (priority, then submission order; duplicates coalesced), each expert's slices kept in
        the planner's rotated order. The reference's planner submits the same experts and
        priorities to its scheduler (comms_planner/expert_parallel.py:266-272)."""
        by_expert: dict[int, list] = {}
        prio: dict[int, int] = {}
        for d in plan.communication_descriptors:
            by_expert.setdefault(int(d.source_expert_id), []).append(d)
            prio.setdefault(int(d.source_expert_id), int(d.priority))
        sched = TransferScheduler()
        for e, p in prio.items():
            sched.submit(e, p)
        sched.close()
        order = []
        while (e := sched.take(0)) is not None:
            order.extend(by_expert[e])
            sched.complete(e)
        return order

    def execute_plan(self, plan, buffer: int | None = None, after_current_stream: bool = True) -> list:
        """Run a communication plan's copies (``DWDPCommunicationPlanner``: 2 MiB slices with
        rotated starts, priorities) into ``buffer`` (default: the next buffer) with ONE call
        into the engine (``dwdp_engine_prefetch_slices``), in ``issue_order``. Returns the
        descriptors in the order they were issued; ``wait_buffer(buffer)`` orders a stream
        after them."""
        buf = self.next_buffer if buffer is None else int(buffer)
        order = self.issue_order(plan)
        arr = (_lib.CopySlice * max(1, len(order)))()
        for i, d in enumerate(order):
            arr[i].expert_id, arr[i].start, arr[i].bytes = int(d.source_expert_id), int(d.start), int(d.count)
        after = torch.cuda.current_stream(self.device_id).cuda_stream if after_current_stream else None
        _chk(_lib.load().dwdp_engine_prefetch_slices(self._eng(), arr, len(order), buf, after), "prefetch_slices")
        for d in order:
            e = int(d.source_expert_id)
            if e not in self._local:
                self._where[e] = buf
        return order

    def wait_buffer(self, buffer: int = 0, stream: torch.cuda.Stream | None = None) -> None:
        s = (stream or torch.cuda.current_stream(self.device_id)).cuda_stream
        _chk(_lib.load().dwdp_engine_wait(self._eng(), buffer, s), "wait")

    # ------------------------------------------------------------------ the reference's form
    @property
    def current_buffer(self) -> int:
        return self._current

    @property
    def next_buffer(self) -> int:
        return (self._current + 1) % max(1, self.num_buffers)

    def prefetch(self, expert_id: int) -> None:
        """Copy a remote expert into the next staging buffer (after the work queued on the
        current stream); local experts need no copy (communication_engine.cpp:85-91)."""
        if int(expert_id) in self._local:
            return
        self.prefetch_into([int(expert_id)], self.next_buffer)

    def wait(self, expert_id: int) -> None:
        """Order the current stream after the copy of ``expert_id`` (communication_engine.cpp:93-96)."""
        e = int(expert_id)
        if e in self._local:
            return
        if e not in self._where:
            raise RuntimeError(f"expert {e} was never prefetched")
        self.wait_buffer(self._where[e])

    def swap_buffers(self) -> None:
        """The next buffer becomes current; what the old current buffer held is no longer
        resident (communication_engine.cpp:128-135). Call it after the compute that read the
        current buffer has been queued."""
        self._eng()
        old = self._current
        self._current = self.next_buffer
        self._where = {e: b for e, b in self._where.items() if b != old}

    def is_resident(self, expert_id: int) -> bool:
        """Local, or staged in the current buffer (communication_engine.cpp:102-105)."""
        e = int(expert_id)
        return e in self._local or self._where.get(e) == self._current

    def get_resident_pointer(self, expert_id: int, buffer: int | None = None) -> int:
        """Device pointer of the usable copy: the local slab, or the staged copy in the current
        buffer (or in ``buffer``). The reference's form waits for the copy on the current
        stream and refuses an expert staged only in the next buffer (communication_engine.cpp:107-126)."""
        e = int(expert_id)
        if buffer is None and e not in self._local:
            if self._where.get(e) == self.next_buffer:
                raise RuntimeError("expert is resident in the next buffer; call swap_buffers after prior compute")
            if e not in self._where:
                raise RuntimeError(f"expert {e} is not resident")
            self.wait(e)
        b = self._current if buffer is None else buffer
        out = ctypes.c_void_p()
        _chk(_lib.load().dwdp_engine_resident_pointer(self._eng(), e, b, ctypes.byref(out)),
             "get_resident_pointer")
        return int(out.value or 0)

    getResidentPointer = get_resident_pointer

    def get_weight(self, expert_id: int) -> int:
        """Device pointer of the expert's weights as usable now (the reference's get_weight):
        the local slab, or the staged copy of a remote expert in the current buffer."""
        return self.get_resident_pointer(expert_id)

    def is_remote(self, expert_id: int) -> bool:
        out = ctypes.c_int(0)
        _chk(_lib.load().dwdp_engine_is_remote(self._eng(), expert_id, ctypes.byref(out)), "is_remote")
        return bool(out.value)

    def set_copy_mode(self, mode: str = "engine", ctas: int = 148) -> None:
        """How prefetches move bytes: ``"engine"`` (cudaMemcpyAsync on the copy engines, the
        default and the reference's mechanism) or ``"sm"`` (one copy kernel of ``ctas`` CTAs
        loading the peer's slabs: faster alone, but it competes with the GEMMs for SMs)."""
        code = {"engine": 0, "sm": 1}.get(mode)
        if code is None:
            raise ValueError(f"copy mode must be 'engine' or 'sm', got {mode!r}")
        _chk(_lib.load().dwdp_engine_set_copy_mode(self._eng(), code, int(ctas)), "set_copy_mode")

    def release(self, expert_id: int) -> None:
        _chk(_lib.load().dwdp_engine_release(self._eng(), expert_id), "release")

    def synchronize(self) -> None:
        _chk(_lib.load().dwdp_engine_synchronize(self._eng()), "synchronize")

    def stats(self) -> dict:
        b, c, s = ctypes.c_ulonglong(0), ctypes.c_ulonglong(0), ctypes.c_void_p()
        _chk(_lib.load().dwdp_engine_stats(self._eng(), ctypes.byref(b), ctypes.byref(c), ctypes.byref(s)), "stats")
        return {"bytes_copied": int(b.value), "copies_issued": int(c.value), "copy_stream": int(s.value or 0)}

    def shutdown(self) -> None:
        if self._h is not None:
            _lib.load().dwdp_engine_destroy(self._h)
            self._h = None

    def __del__(self) -> None:
        try:
            self.shutdown()
        except Exception:  # noqa: BLE001 - interpreter teardown
            pass
