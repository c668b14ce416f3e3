"""ORACLE — test infrastructure only: a plain restatement of the reference's
GPT-2 byte-level BPE tokenizer (src/tokenizer/tokenizer.cc) for checking the
product's own implementation.  Only tests/ import it.

The reference compiles the OLMo pre-split pattern with PCRE2 (UTF and UCP,
tokenizer.cc:15-17, 112-118) and searches it left to right, each search
starting where the previous match ended (tokenizer.cc:165-186); here the same
pattern runs through the `regex` module's finditer, with PCRE2's UCP meaning
of \\s written out (tab .. carriage return and the Z separators).  The merge
loop rescans every adjacent pair per merge (tokenizer.cc:129-157) and the
decoder reads vocabulary strings with the reference's byte rules
(tokenizer.cc:33-48, 188-200).  Parity with PCRE2 itself is unpinned: neither
PCRE2's headers nor ggml's gguf reader exist here, so the reference tokenizer
cannot be built.
"""
from __future__ import annotations

import regex

SPACE = r"[\t\n\x0b\x0c\r\p{Z}]"
NOT_SPACE = r"[^\t\n\x0b\x0c\r\p{Z}]"
PATTERN = regex.compile(
    r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\t\n\x0b\x0c\r\p{Z}\p{L}\p{N}]+|" + SPACE + r"+(?!" +
    NOT_SPACE + r")")


def byte_table() -> list[int]:
    """GPT-2's byte -> code point table (tokenizer.cc:51-65)."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    cps, extra = [0] * 256, 0
    for b in range(256):
        if b in keep:
            cps[b] = b
        else:
            cps[b] = 256 + extra
            extra += 1
    return cps


def split(text: str) -> list[tuple[int, int]]:
    """[begin, end) byte offsets of the pre-split chunks."""
    out = []
    for m in PATTERN.finditer(text):
        out.append((len(text[:m.start()].encode()), len(text[:m.end()].encode())))
    return out


class OracleTokenizer:
    def __init__(self, vocab: list[str], merges: list[str]):
        self.vocab = vocab
        self.ids: dict[str, int] = {}
        for i, t in enumerate(vocab):
            self.ids.setdefault(t, i)
        self.rank: dict[str, int] = {}
        for i, m in enumerate(merges):
            self.rank.setdefault(m, i)
        cps = byte_table()
        self.byte_char = [chr(c) for c in cps]
        self.char_byte = {c: b for b, c in enumerate(cps)}

    def encode_chunk(self, chunk: bytes) -> list[int]:
        syms = [self.byte_char[b] for b in chunk]
        while len(syms) > 1:
            best, best_rank = -1, None
            for i in range(len(syms) - 1):
                r = self.rank.get(syms[i] + " " + syms[i + 1])
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best < 0:
                break
            syms[best:best + 2] = [syms[best] + syms[best + 1]]
        return [self.ids[s] for s in syms if s in self.ids]

    def encode(self, text: str) -> list[int]:
        raw = text.encode()
        out: list[int] = []
        for a, b in split(text):
            out += self.encode_chunk(raw[a:b])
        return out

    def decode(self, ids: list[int]) -> bytes:
        out = bytearray()
        for i in ids:
            if not 0 <= i < len(self.vocab):
                continue
            t = self.vocab[i].encode("utf-8", errors="surrogatepass")
            k = 0
            while k < len(t):
                c = t[k]
                cp, n = c, 1
                if c >> 5 == 0x6 and k + 1 < len(t):
                    cp, n = ((c & 0x1F) << 6) | (t[k + 1] & 0x3F), 2
                elif c >> 4 == 0xE and k + 2 < len(t):
                    cp, n = ((c & 0x0F) << 12) | ((t[k + 1] & 0x3F) << 6) | (t[k + 2] & 0x3F), 3
                k += n
                if cp in self.char_byte:
                    out.append(self.char_byte[cp])
        return bytes(out)
