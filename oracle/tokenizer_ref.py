"""Python restatement of the reference's BPE tokenizer (src/tokenizer.rs:18-178).

TEST INFRASTRUCTURE ONLY: tests/test_tokenizer_native.py compares the library's C++
tokenizer (ab_bpe_*) with this line-by-line restatement of the reference loop (it rescans
every adjacent pair after each merge, as src/tokenizer.rs:131-154 does). The product
package never imports it.
"""
from __future__ import annotations

import bisect
import struct
from typing import List, Optional

BOS_ID = 1  # src/tokenizer.rs:8
EOS_ID = 2


def _parse_byte_token(piece: str) -> Optional[int]:
    """`<0xNN>` byte pieces (src/tokenizer.rs:174-177): u8::from_str_radix(rest, 16), i.e.
    an optional '+' then hex digits whose value fits a byte."""
    if not (piece.startswith("<0x") and piece.endswith(">") and len(piece) > 4):
        return None
    rest = piece[3:-1]
    if rest.startswith("+"):
        rest = rest[1:]
    if not rest or any(c not in "0123456789abcdefABCDEF" for c in rest):
        return None
    v = int(rest, 16)
    return v if v <= 255 else None


class BpeTokenizer:
    """SentencePiece-style BPE from llama2.c `tokenizer.bin` (src/tokenizer.rs:18-178)."""

    def __init__(self, vocab: List[str], vocab_scores: List[float], max_token_length: int):
        if len(vocab) != len(vocab_scores):
            raise ValueError("vocab and scores differ in length")
        self.vocab = list(vocab)
        self.vocab_scores = [float(s) for s in vocab_scores]
        self._max_token_length = int(max_token_length)
        pairs = sorted(((s, i) for i, s in enumerate(self.vocab)), key=lambda p: p[0])
        self._keys = [p[0] for p in pairs]
        self._ids = [p[1] for p in pairs]

    @classmethod
    def from_parts(cls, vocab, vocab_scores, max_token_length) -> "BpeTokenizer":
        return cls(vocab, vocab_scores, max_token_length)

    @classmethod
    def from_path(cls, path: str, vocab_size: int) -> "BpeTokenizer":
        """llama2.c layout: u32 max_token_length, then per piece f32 score, i32 len, bytes."""
        with open(path, "rb") as f:
            data = f.read()
        off = 0

        def take(n):
            nonlocal off
            if off + n > len(data):
                raise ValueError(f"tokenizer file truncated at byte {off}")
            b = data[off:off + n]
            off += n
            return b

        (max_len,) = struct.unpack("<I", take(4))
        vocab, scores = [], []
        for i in range(vocab_size):
            (score,) = struct.unpack("<f", take(4))
            (n,) = struct.unpack("<i", take(4))
            if n < 0:
                raise ValueError(f"tokenizer piece {i} has negative length {n}")
            vocab.append(take(n).decode("utf-8", errors="replace"))
            scores.append(score)
        return cls(vocab, scores, max_len)

    def max_token_length(self) -> int:
        return self._max_token_length

    @staticmethod
    def bos_id() -> int:
        return BOS_ID

    @staticmethod
    def eos_id() -> int:
        return EOS_ID

    def _lookup(self, s: str) -> Optional[int]:
        i = bisect.bisect_left(self._keys, s)
        if i < len(self._keys) and self._keys[i] == s:
            return self._ids[i]
        return None

    def vocab_size(self) -> int:
        return len(self.vocab)

    def encode(self, text: str, bos: bool, eos: bool) -> List[int]:
        """src/tokenizer.rs:101-160: BOS, dummy-prefix space, per-codepoint lookup with
        byte fallback (+3), then greedy highest-score pair merges."""
        tokens: List[int] = []
        if bos:
            tokens.append(BOS_ID)
        if text:
            dummy = self._lookup(" ")
            if dummy is not None:
                tokens.append(dummy)
        raw = text.encode("utf-8")
        i = 0
        while i < len(raw):
            start = i
            i += 1
            while i < len(raw) and (raw[i] & 0xC0) == 0x80 and i - start < 4:
                i += 1
            piece = raw[start:i]
            try:
                s = piece.decode("utf-8")
            except UnicodeDecodeError:
                s = None
            if s is not None:
                tid = self._lookup(s)
                if tid is not None:
                    tokens.append(tid)
                    continue
            tokens.extend(b + 3 for b in piece)
        while True:
            best_score, best_id, best_idx = -1e10, -1, None
            for k in range(max(len(tokens) - 1, 0)):
                merged = self.vocab[tokens[k]] + self.vocab[tokens[k + 1]]
                tid = self._lookup(merged)
                if tid is not None and self.vocab_scores[tid] > best_score:
                    best_score, best_id, best_idx = self.vocab_scores[tid], tid, k
            if best_idx is None:
                break
            tokens[best_idx] = best_id
            del tokens[best_idx + 1]
        if eos:
            tokens.append(EOS_ID)
        return tokens

    def decode(self, prev_token: int, token: int) -> str:
        """src/tokenizer.rs:162-172."""
        piece = self.vocab[token] if 0 <= token < len(self.vocab) else ""
        if prev_token == BOS_ID and piece.startswith(" "):
            piece = piece[1:]
        b = _parse_byte_token(piece)
        if b is not None:
            return chr(b)
        return piece
