"""GBNF grammar engine (CPU)."""
import json

import pytest

from air_rs.structured.gbnf import GbnfConstraint, GbnfGrammar, GbnfState, GbnfError


def _accepts(src, s):
    st = GbnfState(GbnfGrammar.parse(src))
    return all(st.push_char(c) for c in s) and st.is_complete()


def test_literals_classes_quantifiers():
    g = 'root ::= "ab" [0-9]+ ("x" | "yz")? tail\ntail ::= [^a-c]*'
    assert _accepts(g, "ab1")
    assert _accepts(g, "ab12yzq!")
    assert not _accepts(g, "ab")
    assert not _accepts(g, "ab1yzb")


def test_multiline_alternatives_and_comments():
    g = '# comment\nroot ::= a\n    | b  # trailing\na ::= "A"\nb ::= "B" "B"'
    assert _accepts(g, "A") and _accepts(g, "BB") and not _accepts(g, "B")


def test_errors():
    with pytest.raises(GbnfError):
        GbnfGrammar.parse('other ::= "x"')
    with pytest.raises(GbnfError):
        GbnfGrammar.parse('root ::= undefined')


@pytest.mark.parametrize("s,ok", [('{"a": [1, 2.5e3, true, null, "x\\n"]}', True), ("[]", True),
                                  ('{"a" 1}', False), ("-0.5", True), ("01", False)])
def test_json_grammar(s, ok):
    c = GbnfConstraint.json_mode(["x"])
    assert (c.state.can_push_str(s) and (c.push_token(s) or c.is_complete())) == ok


def test_token_mask_and_choice():
    vocab = ["yes", "no", "y", "es", "maybe", "n", "o", "!"]
    c = GbnfConstraint.choice(["yes", "no"], vocab)
    m = c.step_mask()
    assert [vocab[i] for i, a in enumerate(m) if a] == ["yes", "no", "y", "n"]
    c.push_token("y")
    m = c.step_mask()
    assert [vocab[i] for i, a in enumerate(m) if a] == ["es"]
    c.push_token("es")
    assert c.is_complete()
    assert GbnfConstraint.integer(vocab).validate_path([], None)


def test_integer_and_identifier_masks():
    vocab = ["-", "12", "a", "_x", "3.5", " "]
    assert GbnfConstraint.integer(vocab).step_mask() == [True, True, False, False, False, False]
    assert GbnfConstraint.identifier(vocab).step_mask() == [False, False, True, True, False, False]


def test_bitmask_packing():
    vocab = [str(i) for i in range(40)]
    c = GbnfConstraint.integer(vocab)
    bm = c.step_bitmask()
    assert bm.shape == (2,)
    bits = [(int(bm[i // 32]) >> (i % 32)) & 1 for i in range(40)]
    assert bits == [1] * 40
