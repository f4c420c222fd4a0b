"""The seeded synthetic story source that stands in for the training corpus."""

import numpy as np

from leo_b200.synthetic import ALPHABET, pack_stories, story_stream


def test_stories_are_deterministic_and_seeded():
    a = story_stream(7, 6, 20, 60)
    b = story_stream(7, 6, 20, 60)
    c = story_stream(8, 6, 20, 60)
    assert a == b
    assert a != c


def test_story_lengths_and_alphabet():
    stories = story_stream(0, 64, 256, 1024)
    assert all(256 <= len(s) <= 1024 for s in stories)
    allowed = set(int(x) for x in ALPHABET)
    assert all(set(s) <= allowed for s in stories)
    text = b"".join(stories)
    # English-like: space is the most frequent symbol, 'e' the most frequent letter.
    counts = np.bincount(np.frombuffer(text, dtype=np.uint8), minlength=256)
    assert counts.argmax() == ord(" ")
    letters = counts[ord("a"):ord("z") + 1]
    assert letters.argmax() == ord("e") - ord("a")


def test_pack_stories_offsets():
    stories = [b"abc", b"", b"hello"]
    data, offsets = pack_stories(stories)
    assert offsets.tolist() == [0, 3, 3, 8]
    assert bytes(data) == b"abchello"
