"""Seeded synthetic byte stories: an order-2 Markov model over printable ASCII.

The alphabet is 0x20-0x7E plus ``\\n`` (96 symbols).  Unigram weights are
hand-set to English-like letter, space and punctuation frequencies; each of the
96 x 96 two-symbol contexts perturbs those weights with a seeded log-normal
factor so the stream has order-2 structure.  The stream stands in for the
short English prose the reference trains on; none of that corpus is used or
reproduced here.
"""

from __future__ import annotations

import numpy as np

ALPHABET = np.array(list(range(0x20, 0x7F)) + [0x0A], dtype=np.uint8)
_INDEX = {int(b): i for i, b in enumerate(ALPHABET)}

# Hand-set relative frequencies (percent-like units).
_LETTERS = {
    "e": 12.0, "t": 9.1, "a": 8.2, "o": 7.5, "i": 7.0, "n": 6.7, "s": 6.3, "h": 6.1, "r": 6.0, "d": 4.3,
    "l": 4.0, "c": 2.8, "u": 2.8, "m": 2.4, "w": 2.4, "f": 2.2, "g": 2.0, "y": 2.0, "p": 1.9, "b": 1.5,
    "v": 1.0, "k": 0.8, "j": 0.15, "x": 0.15, "q": 0.1, "z": 0.07,
}


def _unigram() -> np.ndarray:
    w = np.full(len(ALPHABET), 0.02, dtype=np.float64)
    for ch, f in _LETTERS.items():
        w[_INDEX[ord(ch)]] = f
        w[_INDEX[ord(ch.upper())]] = f * 0.04
    w[_INDEX[ord(" ")]] = 19.0
    w[_INDEX[ord(".")]] = 1.1
    w[_INDEX[ord(",")]] = 1.0
    w[_INDEX[ord("'")]] = 0.3
    w[_INDEX[ord('"')]] = 0.4
    w[_INDEX[ord("!")]] = 0.1
    w[_INDEX[ord("?")]] = 0.1
    w[_INDEX[ord("\n")]] = 0.3
    for d in "0123456789":
        w[_INDEX[ord(d)]] = 0.05
    return w / w.sum()


class MarkovAscii:
    """Order-2 Markov byte source; ``table[a, b]`` is the CDF of the next symbol."""

    def __init__(self, seed: int = 0, sharpness: float = 1.25):
        rng = np.random.default_rng(np.random.SeedSequence([0x4C454F, seed]))
        base = np.log(_unigram())
        n = len(ALPHABET)
        logits = base[None, None, :] + sharpness * rng.standard_normal((n, n, n))
        space = _INDEX[ord(" ")]
        logits[:, space, space] -= 6.0  # few double spaces
        for p in (".", ",", "!", "?"):
            logits[:, _INDEX[ord(p)], space] += 3.0  # punctuation is usually followed by a space
        probs = np.exp(logits - logits.max(axis=2, keepdims=True))
        probs /= probs.sum(axis=2, keepdims=True)
        self.cdf = np.cumsum(probs, axis=2)
        self.cdf[:, :, -1] = 1.0
        self.rng = np.random.default_rng(np.random.SeedSequence([0x53544F, seed]))

    def stories(self, count: int, min_bytes: int, max_bytes: int) -> list[bytes]:
        lengths = self.rng.integers(min_bytes, max_bytes + 1, size=count)
        total = int(lengths.max()) if count else 0
        out = np.empty((count, total), dtype=np.int64)
        a = np.full(count, _INDEX[ord("\n")], dtype=np.int64)
        b = np.full(count, _INDEX[ord(" ")], dtype=np.int64)
        for pos in range(total):
            u = self.rng.random(count)
            rows = self.cdf[a, b]
            nxt = (rows < u[:, None]).sum(axis=1)
            nxt = np.minimum(nxt, len(ALPHABET) - 1)
            out[:, pos] = nxt
            a, b = b, nxt
        sym = ALPHABET[out]
        return [bytes(sym[i, : int(lengths[i])]) for i in range(count)]


def story_stream(seed: int, count: int, min_bytes: int, max_bytes: int) -> list[bytes]:
    """``count`` stories with lengths uniform in ``[min_bytes, max_bytes]``."""
    return MarkovAscii(seed).stories(count, min_bytes, max_bytes)


def pack_stories(stories: list[bytes]) -> tuple[np.ndarray, np.ndarray]:
    """Concatenate stories into (bytes u8, offsets u64[len+1])."""
    offsets = np.zeros(len(stories) + 1, dtype=np.uint64)
    offsets[1:] = np.cumsum([len(s) for s in stories])
    data = np.frombuffer(b"".join(stories), dtype=np.uint8).copy() if stories else np.zeros(0, np.uint8)
    return data, offsets
