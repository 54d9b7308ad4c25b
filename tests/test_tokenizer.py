"""GGUF BPE tokenizer semantics (merge-all-occurrences, byte fallback)."""
from air_rs.tokenizer import Tokenizer, bytes_to_unicode


def _naive_encode(tok: Tokenizer, text: str):
    """Direct restatement of the reference loop (src/tokenizer.rs:136-212)."""
    sym = tok._symbols(text)
    while True:
        best, pos = None, None
        for i in range(len(sym) - 1):
            r = tok.merge_rank.get((sym[i], sym[i + 1]))
            if r is not None and (best is None or r < best):
                best, pos = r, i
        if best is None:
            break
        a, b = sym[pos], sym[pos + 1]
        i = 0
        while i + 1 < len(sym):
            if sym[i] == a and sym[i + 1] == b:
                sym[i] = a + b
                del sym[i + 1]
            else:
                i += 1
    return [tok._id_of(s) for s in sym]


def _vocab():
    b2c, _ = bytes_to_unicode()
    toks = [b2c[i] for i in range(256)]
    merges = ["Ġ t", "h e", "Ġt he", "a a", "aa a", "i n", "Ġ in", "e r"]
    for m in merges:
        a, b = m.split(" ")
        toks.append(a + b)
    toks += ["<s>", "</s>"]
    return Tokenizer(toks, merges, bos_id=len(toks) - 2, eos_id=len(toks) - 1)


def test_byte_level_detect_and_roundtrip():
    t = _vocab()
    assert t.is_byte_level
    for s in ["the thin herring", "aaaaaaa", "héllo wörld ✓", " in in inner"]:
        ids = t.encode(s)
        assert ids == _naive_encode(t, s)
        assert t.decode(ids) == s


def test_heap_merge_equals_naive_on_random_text():
    import random
    t = _vocab()
    rng = random.Random(0)
    for _ in range(200):
        s = "".join(rng.choice("athe inr") for _ in range(rng.randint(0, 40)))
        assert t.encode(s) == _naive_encode(t, s)


def test_sentencepiece_style_and_byte_fallback():
    toks = ["<unk>", "<s>", "</s>", "▁hi", "h", "i", "▁"] + [f"<0x{i:02X}>" for i in range(256)]
    t = Tokenizer(toks, ["▁ h", "▁h i"], bos_id=1, eos_id=2)
    assert not t.is_byte_level
    assert t.decode([3]) == " hi"
    ids = t.encode("z")
    assert ids == [toks.index("<0x7A>")]
