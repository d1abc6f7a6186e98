"""Tokenizer trait and llama2.c-compatible BPE (src/tokenizer.rs).

Host-only, off the timed decode path. ``BpeTokenizer`` runs the library's C++ tokenizer
(ab_bpe_*: the reference's results with O(n log n) merges). ``sample_argmax`` is the greedy
pick of the decode loop (src/tokenizer.rs:179-189).
"""
from __future__ import annotations

from typing import List, Protocol, Sequence

BOS_ID = 1  # src/tokenizer.rs:8
EOS_ID = 2


class Tokenizer(Protocol):
    def vocab_size(self) -> int: ...

    def encode(self, text: str, bos: bool, eos: bool) -> List[int]: ...

    def decode(self, prev_token: int, token: int) -> str: ...


def sample_argmax(logits: Sequence[float]) -> int:
    """First index of the maximum (ties go to the lowest index)."""
    max_i = 0
    max_p = logits[0]
    for i in range(1, len(logits)):
        p = logits[i]
        if p > max_p:
            max_i = i
            max_p = p
    return int(max_i)


class BpeTokenizer:
    """SentencePiece-style BPE from llama2.c `tokenizer.bin` (src/tokenizer.rs:18-178), run
    by the C++ host library (ab_bpe_*): the reference's encode/decode results, with
    O(n log n) merges (a linked list of symbols and a lazily invalidated max-heap of
    candidate pairs) where the reference rescans every pair after each merge."""

    def __init__(self, handle):
        self._h = handle
        from . import _abi

        self._abi = _abi
        vs, ml = _abi.C.c_uint32(), _abi.C.c_uint32()
        _check_native(_abi.lib().ab_bpe_info(self._h, _abi.C.byref(vs), _abi.C.byref(ml)))
        self._vocab_size, self._max_token_length = int(vs.value), int(ml.value)

    @classmethod
    def from_path(cls, path: str, vocab_size: int) -> "BpeTokenizer":
        import os

        from . import _abi

        h = _abi.C.c_void_p()
        _check_native(_abi.lib().ab_bpe_from_path(os.fsencode(path), int(vocab_size),
                                                  _abi.C.byref(h)))
        return cls(h)

    @classmethod
    def from_parts(cls, vocab, vocab_scores, max_token_length) -> "BpeTokenizer":
        from . import _abi

        C = _abi.C
        raw = [v.encode("utf-8") if isinstance(v, str) else bytes(v) for v in vocab]
        if len(raw) != len(vocab_scores):
            raise ValueError("vocab and scores differ in length")
        n = len(raw)
        pieces = (C.c_char_p * max(n, 1))(*raw)
        lens = (C.c_uint32 * max(n, 1))(*[len(b) for b in raw])
        scores = (C.c_float * max(n, 1))(*[float(s) for s in vocab_scores])
        h = C.c_void_p()
        _check_native(_abi.lib().ab_bpe_from_parts(pieces, lens, scores, n,
                                                   int(max_token_length), C.byref(h)))
        return cls(h)

    def vocab_size(self) -> int:
        return self._vocab_size

    def max_token_length(self) -> int:
        return self._max_token_length

    @staticmethod
    def bos_id() -> int:
        return BOS_ID

    @staticmethod
    def eos_id() -> int:
        return EOS_ID

    def encode(self, text: str, bos: bool, eos: bool) -> List[int]:
        C = self._abi.C
        raw = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        n = C.c_uint32()
        cap = len(raw) + 3
        out = (C.c_int32 * cap)()
        _check_native(self._abi.lib().ab_bpe_encode(self._h, raw, len(raw), int(bos), int(eos),
                                                    out, cap, C.byref(n)))
        return list(out[:n.value])

    def decode(self, prev_token: int, token: int) -> str:
        C = self._abi.C
        n = C.c_uint32()
        _check_native(self._abi.lib().ab_bpe_decode(self._h, int(prev_token), int(token), None,
                                                    0, C.byref(n)))
        buf = C.create_string_buffer(max(n.value, 1))
        _check_native(self._abi.lib().ab_bpe_decode(self._h, int(prev_token), int(token), buf,
                                                    n.value, C.byref(n)))
        return buf.raw[:n.value].decode("utf-8")

    def close(self):
        if getattr(self, "_h", None):
            self._abi.lib().ab_bpe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_native(status: int):
    if status:
        from . import _check

        _check(status)


# the name the first version of this package exported for the C++ tokenizer
NativeBpeTokenizer = BpeTokenizer
