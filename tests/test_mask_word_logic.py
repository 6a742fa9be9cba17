"""CPU check of the word-level mask composition used by mask_build_kernel
(fftsparse_b200/csrc/mask.cu): the sink / recent / local / causal terms as
low- or high-bit masks and the stripe head's selected lags as one bit-reversed
32-bit window of the lag bit array, against the per-bit rule of the reference's
prior mask and mask union (my_attn_v7.py:95, :560, :612, :641; the canonical
restatement in oracle/ffts_oracle.c).  Random parameters, every (row, word) of small N."""
import random

import pytest

M32 = 0xFFFFFFFF


def bits_below(x):
    return 0 if x <= 0 else (M32 if x >= 32 else (1 << x) - 1)


def lag_window(words, base):
    W = len(words)
    wlo, sh = base >> 5, base & 31  # Python >> floors like the kernel's arithmetic shift
    a = words[wlo] if 0 <= wlo < W else 0
    b = words[wlo + 1] if 0 <= wlo + 1 < W else 0
    return ((a >> sh) | (b << (32 - sh))) & M32 if sh else a


def brev(x):
    return int(f"{x:032b}"[::-1], 2)


def word_rule(i, w, N, p, lag_words, lag_on, extra):
    j0 = 32 * w
    word = bits_below(p["keep_sink"] - j0) | (~bits_below(N - p["keep_recent"] - j0) & M32) | \
        (~bits_below(i - p["local_window"] - j0) & M32)
    if lag_on:
        lagw = brev(lag_window(lag_words, i - j0 - 31))
        word |= lagw & bits_below(i - p["remote_start"] + 1 - j0) & (~bits_below(p["keep_sink"] - j0) & M32)
    word |= extra
    return word & bits_below(i + 1 - j0)


def bit_rule(i, w, N, p, lag_bits, lag_on, extra):
    word = 0
    for t in range(32):
        j = 32 * w + t
        if j > i:
            break
        tau = i - j
        on = j < p["keep_sink"] or j >= N - p["keep_recent"] or tau <= p["local_window"]
        if lag_on:
            on |= tau >= p["remote_start"] and lag_bits[tau] and j >= p["keep_sink"]
        on |= bool((extra >> t) & 1)
        word |= int(on) << t
    return word


@pytest.mark.parametrize("seed", range(12))
def test_word_rule_equals_bit_rule(seed):
    rng = random.Random(seed)
    N = rng.choice([10, 31, 32, 33, 64, 95, 130, 257])
    W = (N + 31) // 32
    p = {"keep_sink": rng.randint(0, N // 4), "keep_recent": rng.randint(0, N // 4),
         "local_window": rng.randint(0, N // 3), "remote_start": rng.randint(0, N)}
    lag_bits = [0] * (32 * W)
    for t in range(p["remote_start"], N):
        lag_bits[t] = int(rng.random() < 0.3)
    lag_words = [sum(lag_bits[32 * w + k] << k for k in range(32)) for w in range(W)]
    for lag_on in (False, True):
        for i in range(N):
            for w in range(W):
                extra = rng.getrandbits(32) if rng.random() < 0.3 else 0
                assert word_rule(i, w, N, p, lag_words, lag_on, extra) == \
                    bit_rule(i, w, N, p, lag_bits, lag_on, extra), (i, w, p, lag_on)
