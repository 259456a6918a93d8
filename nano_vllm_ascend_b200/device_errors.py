"""Device-side errors of the hot-path kernels, raised on the host.

The kernels never fault on bad metadata: a block id outside the pool is read
as zeros, a slot outside the pool is skipped, a context longer than its
block-table row is clamped, and each sets a bit in an int32 error word (the
bits are listed in csrc/nvk_common.cuh). This module turns those bits into
the exceptions the reference raises for the same inputs:

* a slot outside the pool -> ``IndexError`` (the reference's
  ``Tensor.index_copy_`` raises it, src/nanovllm_ascend/npu/paged_kv_cache.py:68-69);
* a context longer than its block-table row -> ``RuntimeError("missing
  block: ...")`` (``BlockManager._physical_slot``,
  src/nanovllm_ascend/npu/block_manager.py:194-205);
* a block id outside the pool, or a bounded device wait that ran out ->
  ``RuntimeError``.

All of them are ``KVCacheDeviceError`` (a ``RuntimeError``; the slot case is
also an ``IndexError``), carrying the raw ``bits``.

Each device has one error word shared by the append and prefill launches of
the drop-in classes; decode launches report into the head of their split-K
workspace, which is registered here. Reading a word needs the stream, so the
drop-ins do it without blocking: after a launch, if no read is in flight, the
words launched since the last read are copied into pinned host memory behind
an event; the next call raises once that copy has landed and shows a bit.
Bits are sticky until raised (the word is then cleared on the stream), so
nothing is lost between reads. ``check_errors()`` reads every word now
(synchronising the current stream) and raises; a step driver calls it once
per step, and ``DecodeGraphRunner`` reads its entry's words after each replay.
Nothing here runs while a stream is capturing.
"""

from __future__ import annotations

import torch

WAIT_TIMEOUT = 1
BAD_BLOCK_ID = 2
BAD_SLOT = 4
CONTEXT_TOO_LONG = 8
PEER_TIMEOUT = 16


class KVCacheDeviceError(RuntimeError):
    """A hot-path kernel flagged bad metadata or a device wait that ran out."""

    def __init__(self, message: str, bits: int):
        super().__init__(message)
        self.bits = bits


class KVSlotIndexError(KVCacheDeviceError, IndexError):
    """A slot_mapping entry outside the pool (the reference's index_copy_ IndexError)."""


def error_for(bits: int, where: str) -> KVCacheDeviceError:
    """The exception for error-word ``bits`` reported by ``where`` (a kernel name)."""
    parts = []
    if bits & BAD_SLOT:
        parts.append("a slot_mapping entry is out of bounds for the KV pool (index_copy_ would raise)")
    if bits & CONTEXT_TOO_LONG:
        parts.append("missing block: a context length exceeds its block-table row")
    if bits & BAD_BLOCK_ID:
        parts.append("a block-table entry is outside the KV pool")
    if bits & WAIT_TIMEOUT:
        parts.append("a bounded device wait ran out (kernel abandoned its work)")
    if bits & PEER_TIMEOUT:
        parts.append("a peer rank's epoch flag did not arrive in time")
    unknown = bits & ~(BAD_SLOT | CONTEXT_TOO_LONG | BAD_BLOCK_ID | WAIT_TIMEOUT | PEER_TIMEOUT)
    if unknown:
        parts.append(f"unknown error bits {unknown:#x}")
    msg = f"{where}: " + "; ".join(parts) + f" (error word {bits:#x})"
    cls = KVSlotIndexError if bits & BAD_SLOT else KVCacheDeviceError
    return cls(msg, bits)


SHARED = "kv append / prefill"


class DeviceErrorState:
    """The error words of one device and the read in flight (see the module docstring).

    Words are keyed by a name that also appears in the raised message; the
    shared append/prefill word is ``SHARED``.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self._words: dict[str, torch.Tensor] = {SHARED: self.word}
        self._dirty: set[str] = set()
        self._inflight: tuple[torch.cuda.Event | None, torch.Tensor, list[str]] | None = None

    def watch(self, name: str, word: torch.Tensor) -> str:
        """Registers (or replaces) the device word called ``name``: the first int32 of
        ``word`` (e.g. a decode workspace, whose head is its error word)."""
        self._words[name] = word.view(torch.int32)[:1]
        return name

    def forget(self, name: str) -> None:
        self._words.pop(name, None)
        self._dirty.discard(name)

    def mark(self, *names: str) -> None:
        """Records that launches wrote these words (default: the shared word) without
        starting a read; the next ``launched`` or ``check`` reads them."""
        self._dirty.update(names or (SHARED,))

    def launched(self, *names: str) -> None:
        """Marks words as written by launches just enqueued on the current stream
        (default: the shared word) and starts a non-blocking read if none is in flight."""
        if torch.cuda.is_current_stream_capturing():
            return
        self._dirty.update(names or (SHARED,))
        self._poll()

    def _poll(self) -> None:
        if self._inflight is not None:
            if not self._inflight[0].query():
                return
            self._raise_from(self._inflight)  # landed: raise before starting the next read
        names = [n for n in self._dirty if n in self._words]
        self._dirty.clear()
        if names:
            host = self._copy_out(names)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._inflight = (ev, host, names)

    def _copy_out(self, names: list[str]) -> torch.Tensor:
        host = torch.empty(len(names), dtype=torch.int32, pin_memory=True)
        for i, n in enumerate(names):
            host[i:i + 1].copy_(self._words[n], non_blocking=True)
        return host

    def _raise_from(self, inflight) -> None:
        _, host, names = inflight
        self._inflight = None
        flagged = [(n, int(v)) for n, v in zip(names, host.tolist()) if v]
        if not flagged:
            return
        bits = 0
        for n, v in flagged:
            bits |= v
            if n in self._words:
                self._words[n].zero_()  # stream-ordered: later launches start clean
        raise error_for(bits, ", ".join(sorted(n for n, _ in flagged)))

    def raise_if_flagged(self) -> None:
        """Raises if a completed read shows an error bit (does not wait)."""
        if torch.cuda.is_current_stream_capturing():
            return
        if self._inflight is not None and self._inflight[0].query():
            self._raise_from(self._inflight)

    def check(self) -> None:
        """Reads every registered word now (waits for the current stream) and raises on any bit."""
        if self._inflight is not None:
            self._inflight[0].synchronize()
            self._raise_from(self._inflight)
        names = list(self._words)
        self._dirty.clear()
        host = self._copy_out(names)
        torch.cuda.current_stream(self.device).synchronize()
        self._raise_from((None, host, names))


_STATES: dict[int, DeviceErrorState] = {}


def state(device: torch.device | None = None) -> DeviceErrorState:
    """The error state of ``device`` (default: the current CUDA device)."""
    idx = torch.cuda.current_device() if device is None or device.index is None else device.index
    st = _STATES.get(idx)
    if st is None:
        st = DeviceErrorState(torch.device("cuda", idx))
        _STATES[idx] = st
    return st


def check_errors(device: torch.device | None = None) -> None:
    """Raises the pending device-side error of ``device``'s hot-path kernels, if any
    (waits for the current stream)."""
    with torch.cuda.device(state(device).device):
        state(device).check()
