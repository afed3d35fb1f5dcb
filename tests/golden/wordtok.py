"""A deterministic stand-in for the HeartMuLa text tokenizer (test infrastructure).

``generate`` takes the caller's tokenizer object and only calls
``tokenizer.encode(text).ids`` (``app/engine.py:357-372``).  This one maps every
whitespace-separated word to a fixed id from its bytes, so the reference's prompt
assembly (lower-casing, ``<tag>`` wrapping, BOS/EOS insertion) can run without the
real tokenizer files.
"""
from __future__ import annotations


class _Enc:
    def __init__(self, ids):
        self.ids = ids


class WordTokenizer:
    def encode(self, text: str) -> _Enc:
        ids = []
        for w in text.split():
            h = 0
            for b in w.encode("utf-8"):
                h = (h * 131 + b) % 1_000_003
            ids.append(1000 + h % 120_000)
        return _Enc(ids)
