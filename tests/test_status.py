"""Host logic of the bounded-wait status words (fftsparse_b200.status), on CPU.

A kernel whose bounded wait runs out stores a nonzero code into a status word
and returns; the operators must turn that into an exception instead of handing
back wrong output silently.  Here the library's attention entry point is
replaced by a stand-in that writes such a code through the pointer it is given,
so the real sparse_attention / myattn_prefill host code runs without a GPU.
"""
import ctypes

import pytest
import torch

import fftsparse_b200.prefill as P
from fftsparse_b200 import status as S


def test_status_word_raises_once_and_clears():
    w = S.StatusWord("cpu")
    w.poll()  # zero: nothing to report
    w.word[0] = 5
    with pytest.raises(S.WaitTimeout) as exc:
        w.poll()
    assert exc.value.code == 5 and "peer" in str(exc.value)
    w.poll()  # cleared by the raise
    w.word[0] = 3
    with pytest.raises(S.WaitTimeout):
        w.check()


class _FakeLib:
    """ffts_sparse_attn_fwd stand-in: the n-th call stores codes[n] into *status."""

    def __init__(self, codes):
        self.codes = list(codes)
        self.calls = 0

    def ffts_sparse_attn_fwd(self, *args):
        status_ptr = args[-2]
        code = self.codes[self.calls] if self.calls < len(self.codes) else 0
        self.calls += 1
        if code:
            ctypes.c_int32.from_address(status_ptr).value = code
        return 0


def test_sparse_attention_surfaces_a_timeout_on_the_next_call(monkeypatch):
    fake = _FakeLib([0, 3, 0, 0])
    monkeypatch.setattr(P._lib, "load", lambda: fake)
    monkeypatch.setattr(P, "_stream_ptr", lambda device: 0)
    S._DEVICE_WORDS.pop(-1, None)
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    bits = torch.full((1, 1, 1, 1), -1, dtype=torch.int32)
    P.sparse_attention(q, q, q, bits, 128)          # call 1: fine
    P.sparse_attention(q, q, q, bits, 128)          # call 2: its kernel "times out"
    with pytest.raises(S.WaitTimeout) as exc:       # call 3 reports it before launching
        P.sparse_attention(q, q, q, bits, 128)
    assert exc.value.code == 3
    assert fake.calls == 2, "the call that reports the time-out must not launch"
    P.sparse_attention(q, q, q, bits, 128)          # the word was cleared: calls go on
    S.check_status("cpu")
    # a caller-supplied status word is the caller's to read: no exception from the operator
    own = torch.zeros(1, dtype=torch.int32)
    fake.codes = [0] * fake.calls + [2]
    P.sparse_attention(q, q, q, bits, 128, status=own)
    P.sparse_attention(q, q, q, bits, 128, status=own)
    assert int(own[0]) == 2


def test_myattn_prefill_dense_branch_uses_the_device_word(monkeypatch):
    fake = _FakeLib([1])
    monkeypatch.setattr(P._lib, "load", lambda: fake)
    monkeypatch.setattr(P, "_stream_ptr", lambda device: 0)
    S._DEVICE_WORDS.pop(-1, None)

    # the operator asserts is_cuda first (as the reference does); a CPU tensor subclass satisfies it
    class Claim(torch.Tensor):
        @property
        def is_cuda(self):
            return True

    x = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16).as_subclass(Claim)
    P.myattn_prefill(x, x, x, 0)  # L < 10 blocks: dense causal branch, "times out"
    with pytest.raises(S.WaitTimeout):
        S.check_status("cpu")
