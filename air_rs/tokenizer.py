"""GGUF BPE tokenizer.

Same semantics as the reference (``src/tokenizer.rs:26-255``): GPT-2 byte->unicode map,
byte-level mode auto-detected by the presence of ``Ġ``/``ĠThe`` in the vocab, encoding by
repeatedly picking the lowest-rank merge among adjacent pairs and merging *all*
occurrences of that pair left to right, ``<0xNN>`` byte fallback for unknown single
symbols (else id 0), SentencePiece ``▁`` -> space on decode for non-byte-level vocabs.
BOS is not added here; callers prepend it (``src/inference_step.rs:32-33``).

The merge loop is implemented with a rank heap over a linked list of symbols so it is
O(n log n) instead of the reference's O(n^2) rescans; the result is identical because
each round still merges every occurrence of the globally lowest-rank pair.
"""
from __future__ import annotations

import heapq
from functools import lru_cache


@lru_cache(maxsize=1)
def bytes_to_unicode() -> tuple[dict[int, str], dict[str, int]]:
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + \
        list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    b2c = {b: chr(c) for b, c in zip(bs, cs)}
    return b2c, {c: b for b, c in b2c.items()}


class Tokenizer:
    def __init__(self, tokens: list[str], merges: list[str] | None = None,
                 bos_id: int = 1, eos_id: int = 2):
        self.id_to_token = list(tokens)
        self.vocab = {t: i for i, t in enumerate(self.id_to_token)}
        self.merge_rank: dict[tuple[str, str], int] = {}
        for i, m in enumerate(merges or []):
            parts = m.split(" ")
            if len(parts) == 2:
                self.merge_rank[(parts[0], parts[1])] = i
        self.byte_to_char, self.char_to_byte = bytes_to_unicode()
        self.is_byte_level = "Ġ" in self.vocab or "ĠThe" in self.vocab
        self.bos_id = bos_id
        self.eos_id = eos_id

    @classmethod
    def from_gguf_metadata(cls, md: dict) -> "Tokenizer":
        toks = md.get("tokenizer.ggml.tokens") or []
        merges = md.get("tokenizer.ggml.merges") or []
        return cls(toks, merges, int(md.get("tokenizer.ggml.bos_token_id", 1)),
                   int(md.get("tokenizer.ggml.eos_token_id", 2)))

    @classmethod
    def byte_vocab(cls, vocab_size: int, bos_id: int = 1, eos_id: int = 2) -> "Tokenizer":
        """A vocab whose first 256 ids are ``<0xNN>`` byte tokens, the rest placeholders."""
        toks = [f"<0x{i:02X}>" for i in range(min(256, vocab_size))]
        toks += [f"<tok{i}>" for i in range(len(toks), vocab_size)]
        return cls(toks, [], bos_id, eos_id)

    def __len__(self):
        return len(self.id_to_token)

    @property
    def vocab_size(self) -> int:
        return len(self.id_to_token)

    def _symbols(self, text: str) -> list[str]:
        if self.is_byte_level:
            return [self.byte_to_char[b] for b in text.encode("utf-8")]
        return list(text)

    def encode(self, text: str) -> list[int]:
        if not text:
            return []
        sym = self._symbols(text)
        n = len(sym)
        nxt = list(range(1, n + 1))
        prv = list(range(-1, n - 1))
        alive = [True] * n
        heap: list[tuple[int, int, str, str]] = []
        rank = self.merge_rank

        def push(i):
            j = nxt[i]
            if j < n:
                r = rank.get((sym[i], sym[j]))
                if r is not None:
                    heapq.heappush(heap, (r, i, sym[i], sym[j]))

        for i in range(n - 1):
            push(i)
        while heap:
            r = heap[0][0]
            # collect every live occurrence of the lowest-rank pair, merge left to right
            batch = []
            while heap and heap[0][0] == r:
                batch.append(heapq.heappop(heap))
            batch.sort(key=lambda e: e[1])
            touched = []
            for _, i, a, b in batch:
                if not alive[i] or sym[i] != a:
                    continue
                j = nxt[i]
                if j >= n or sym[j] != b:
                    continue
                sym[i] = a + b
                alive[j] = False
                nxt[i] = nxt[j]
                if nxt[j] < n:
                    prv[nxt[j]] = i
                touched.append(i)
            for i in touched:
                if alive[i]:
                    push(i)
                    if prv[i] >= 0 and alive[prv[i]]:
                        push(prv[i])
        out = []
        i = 0
        while i < n:
            if alive[i]:
                out.append(self._id_of(sym[i]))
            i = nxt[i] if alive[i] else i + 1
        return out

    def _id_of(self, s: str) -> int:
        t = self.vocab.get(s)
        if t is not None:
            return t
        if len(s) == 1:
            b = self.char_to_byte.get(s)
            if b is not None:
                return self.vocab.get(f"<0x{b:02X}>", 0)
        return 0

    def _raw_to_text(self, raw: str) -> str:
        if self.is_byte_level:
            bs = bytes(self.char_to_byte[c] for c in raw if c in self.char_to_byte)
            return bs.decode("utf-8", errors="replace")
        return raw.replace("▁", " ")

    @staticmethod
    def _byte_piece(tok: str) -> int | None:
        """SentencePiece byte-fallback token ``<0xNN>`` -> NN (else None)."""
        if len(tok) == 6 and tok.startswith("<0x") and tok.endswith(">"):
            try:
                return int(tok[3:5], 16)
            except ValueError:
                return None
        return None

    def decode(self, ids: list[int]) -> str:
        toks = [self.id_to_token[i] for i in ids if 0 <= i < len(self.id_to_token)]
        if self.is_byte_level:
            return self._raw_to_text("".join(toks))
        # byte-fallback pieces are reassembled into UTF-8 (the reference prints them verbatim)
        out, pending = [], bytearray()
        for t in toks:
            b = self._byte_piece(t)
            if b is not None:
                pending.append(b)
                continue
            if pending:
                out.append(pending.decode("utf-8", errors="replace"))
                pending = bytearray()
            out.append(t.replace("▁", " "))
        if pending:
            out.append(pending.decode("utf-8", errors="replace"))
        return "".join(out)

    def decode_token(self, i: int) -> str:
        raw = self.id_to_token[i] if 0 <= i < len(self.id_to_token) else "<unk>"
        if not self.is_byte_level:
            b = self._byte_piece(raw)
            if b is not None:
                return chr(b) if b < 0x80 else bytes([b]).decode("latin-1")
        return self._raw_to_text(raw)

    def token_texts(self) -> list[str]:
        return [self.decode_token(i) for i in range(len(self.id_to_token))]
