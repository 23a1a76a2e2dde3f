"""Long-audio chunking for the ASR cascade: overlapping windows and seam-aware merging.

A backend with a fixed input window still handles long clips: the waveform is
cut into windows of ``window_s`` seconds that overlap by ``overlap_s`` seconds
(a hard cut can split a word, so the overlap is transcribed twice), and the
per-window transcripts are joined with the duplicated words at each seam
removed. Behaviour follows the reference's chunker
(src/granite_switch/vllm/audio/chunking.py:23-92): windows advance by
``window_s - overlap_s``, a clip no longer than one window is one segment,
and a seam drops the longest run of words (up to 60) that ends the text so
far and starts the next window, compared without case or punctuation.
"""
from __future__ import annotations

import re

import numpy as np

SEAM_SEARCH_WORDS = 60
_NON_WORD = re.compile(r"[^\w]+")


def split_waveform(samples: np.ndarray, sr: int, window_s: float, overlap_s: float) -> list[np.ndarray]:
    """Overlapping windows of a mono waveform, in order (views, no copies)."""
    if window_s <= 0:
        raise ValueError(f"window_s must be > 0, got {window_s}")
    if not 0 <= overlap_s < window_s:
        raise ValueError(f"overlap_s must satisfy 0 <= overlap_s < window_s; got overlap_s={overlap_s}, "
                         f"window_s={window_s}")
    win = max(1, int(round(window_s * sr)))
    hop = max(1, int(round((window_s - overlap_s) * sr)))
    n = len(samples)
    if n <= win:
        return [samples]
    starts = list(range(0, max(n - win, 0) + hop, hop))
    # the last window ends at (or past) the end of the clip; drop starts past it
    out, last_end = [], 0
    for s in starts:
        if last_end >= n:
            break
        out.append(samples[s:s + win])
        last_end = s + win
    return out


def _key(word: str) -> str:
    return _NON_WORD.sub("", word).lower()


def seam_overlap(prev: list[str], nxt: list[str], limit: int = SEAM_SEARCH_WORDS) -> int:
    """Longest ``k <= limit`` with ``prev[-k:] == nxt[:k]`` (case / punctuation insensitive)."""
    k_max = min(len(prev), len(nxt), limit)
    if k_max == 0:
        return 0
    tail = [_key(w) for w in prev[-k_max:]]
    head = [_key(w) for w in nxt[:k_max]]
    for k in range(k_max, 0, -1):
        if tail[k_max - k:] == head[:k]:
            return k
    return 0


def merge_transcripts(texts: list[str]) -> str:
    """Join per-window transcripts, keeping one copy of the words at each seam."""
    words: list[str] = []
    for text in texts:
        cur = text.split()
        if not cur:
            continue
        if words:
            cur = cur[seam_overlap(words, cur):]
        words.extend(cur)
    return " ".join(words)


__all__ = ["split_waveform", "merge_transcripts", "seam_overlap", "SEAM_SEARCH_WORDS"]
