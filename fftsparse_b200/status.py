"""Status words of the kernels' bounded waits, read back without stalling the stream.

Every wait inside the attention and QKV projection kernels and the peer all-gather is
bounded; when
one runs out the kernel stores a nonzero code into a status word in device
memory and returns instead of hanging (the output it leaves is then wrong).
The reference has no such failure mode (its kernels come from a library whose
waits are unbounded), so the codes are this library's own:

  1  attention: the TMA producer's wait timed out
  2  attention: the MMA issuer's wait timed out
  3  attention: a softmax warp's wait timed out
  4  attention: dynamic shared memory was not 1024-byte aligned (nothing ran)
  5  peer all-gather: a peer's epoch flag never arrived
  6  QKV projection: the TMA producer's wait timed out
  7  QKV projection: the MMA issuer's wait timed out
  8  QKV projection: an epilogue warp's wait timed out
  9  QKV projection: dynamic shared memory was not 1024-byte aligned (nothing ran)

A ``StatusWord`` owns one such word.  After each launch that may write it,
``read_back`` enqueues an asynchronous copy of the word into pinned host memory
on the launching stream; ``poll`` (called before the next launch) raises
``WaitTimeout`` once such a copy has landed with a nonzero code, and never
blocks.  So a time-out surfaces as an exception at the first call after the
failing kernel has completed.  ``check`` synchronises the device and raises at
once; call it (``fftsparse_b200.check_status()``) where the result must be
known to be good, e.g. at the end of a forward pass.  The word is sticky (a
kernel only ever sets it), so a read that overtakes an earlier one loses
nothing; raising clears it.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

__all__ = ["WaitTimeout", "StatusWord", "device_status", "check_status"]

MESSAGES = {
    1: "attention kernel: the TMA producer's bounded wait timed out",
    2: "attention kernel: the MMA issuer's bounded wait timed out",
    3: "attention kernel: a softmax warp's bounded wait timed out",
    4: "attention kernel: dynamic shared memory was not 1024-byte aligned (nothing ran)",
    5: "peer all-gather: a peer's epoch flag never arrived (its rows are missing)",
    6: "QKV projection kernel: the TMA producer's bounded wait timed out",
    7: "QKV projection kernel: the MMA issuer's bounded wait timed out",
    8: "QKV projection kernel: an epilogue warp's bounded wait timed out",
    9: "QKV projection kernel: dynamic shared memory was not 1024-byte aligned (nothing ran)",
}


class WaitTimeout(RuntimeError):
    """A kernel's bounded wait ran out; the output of that call is not valid."""

    def __init__(self, code: int):
        super().__init__(f"{MESSAGES.get(code, 'unknown status')} [status {code}]")
        self.code = code


class StatusWord:
    """One int32 status word on ``device`` with an asynchronous host read-back."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._cuda = self.device.type == "cuda"
        self._host = torch.zeros(1, dtype=torch.int32, pin_memory=True) if self._cuda else None
        self._event: Optional[torch.cuda.Event] = None

    def read_back(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue the copy of the word to the host after the work already on ``stream``."""
        if not self._cuda:
            return
        stream = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(stream):
            self._host.copy_(self.word, non_blocking=True)
        if self._event is None:
            self._event = torch.cuda.Event()
        self._event.record(stream)

    def poll(self) -> None:
        """Raise WaitTimeout if a completed read-back holds a nonzero code (never blocks)."""
        if not self._cuda:
            code = int(self.word[0])
        elif self._event is None or not self._event.query():
            return
        else:
            code = int(self._host[0])
        if code:
            self._raise(code)

    def check(self) -> None:
        """Wait for the device and raise WaitTimeout if the word is nonzero."""
        if self._cuda:
            torch.cuda.synchronize(self.device)
        code = int(self.word[0].item())
        if code:
            self._raise(code)

    def _raise(self, code: int) -> None:
        self.word.zero_()
        if self._host is not None:
            self._host.zero_()
        self._event = None
        raise WaitTimeout(code)


_DEVICE_WORDS: Dict[int, StatusWord] = {}


def device_status(device) -> StatusWord:
    """The status word the operators use on ``device`` when the caller passes none."""
    device = torch.device(device)
    if device.type != "cuda":  # host-side tests drive the operators' logic with CPU tensors
        idx, dev = -1, torch.device("cpu")
    else:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        dev = torch.device("cuda", idx)
    word = _DEVICE_WORDS.get(idx)
    if word is None:
        word = StatusWord(dev)
        _DEVICE_WORDS[idx] = word
    return word


def check_status(device=None) -> None:
    """Synchronise ``device`` (default: every device used so far) and raise
    WaitTimeout if any of the operators' calls there had a bounded wait time out."""
    if device is not None:
        device_status(device).check()
        return
    for word in list(_DEVICE_WORDS.values()):
        word.check()
