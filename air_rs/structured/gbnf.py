"""GBNF grammar-constrained decoding.

Same feature set as the reference (``src/gbnf.rs``): a GBNF parser (rules ``name ::= ...``,
string literals with escapes, character classes with ranges / negation, rule references,
groups, ``*``/``+``/``?`` quantifiers, ``#`` comments, a mandatory ``root`` rule), a
character-level recogniser (``can_push_str`` / ``push_char`` / ``is_complete``) and
``GbnfConstraint`` with the builders ``json_mode`` / ``integer`` / ``identifier`` / ``choice``
plus ``step_mask`` / ``apply_to_logits`` / ``push_token`` / ``validate_path``.

The recogniser is a set of pushdown stacks over compiled alternatives (each stack is a
tuple of element positions, the top being the next element to match), expanded eagerly
through rule references. Token masks walk a trie of the vocabulary's token texts once per
step, pruning every branch whose prefix the grammar rejects, instead of re-simulating each
of the ~10^5 token strings independently as the reference does.
"""
from __future__ import annotations

import functools
from dataclasses import dataclass

import torch


class GbnfError(ValueError):
    pass


# ---------------------------------------------------------------------------
# parsing
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class CharSet:
    ranges: tuple[tuple[int, int], ...]
    negated: bool = False

    def match(self, c: int) -> bool:
        hit = any(lo <= c <= hi for lo, hi in self.ranges)
        return hit != self.negated


@dataclass(frozen=True)
class Ref:
    rule: int


END = None  # marks the end of an alternative


class _Parser:
    def __init__(self, src: str):
        self.src = src
        self.i = 0
        self.names: dict[str, int] = {}
        self.rules: list[list[list]] = []   # rule -> alternatives -> elements

    def err(self, msg):
        line = self.src.count("\n", 0, self.i) + 1
        raise GbnfError(f"GBNF parse error at line {line}: {msg}")

    def rule_id(self, name: str) -> int:
        if name not in self.names:
            self.names[name] = len(self.rules)
            self.rules.append(None)
        return self.names[name]

    def new_rule(self, alts) -> int:
        self.rules.append(alts)
        return len(self.rules) - 1

    def ws(self, newlines=True):
        while self.i < len(self.src):
            ch = self.src[self.i]
            if ch == "#":
                while self.i < len(self.src) and self.src[self.i] != "\n":
                    self.i += 1
            elif ch in " \t\r" or (newlines and ch == "\n"):
                self.i += 1
            else:
                break

    def name(self) -> str:
        j = self.i
        while self.i < len(self.src) and (self.src[self.i].isalnum() or self.src[self.i] in "-_"):
            self.i += 1
        if j == self.i:
            self.err("expected a rule name")
        return self.src[j:self.i]

    def char(self) -> int:
        ch = self.src[self.i]
        if ch == "\\":
            self.i += 1
            if self.i >= len(self.src):
                self.err("dangling escape")
            e = self.src[self.i]
            self.i += 1
            simple = {"n": 10, "t": 9, "r": 13, "\\": 92, '"': 34, "[": 91, "]": 93, "-": 45, "'": 39}
            if e in simple:
                return simple[e]
            if e in "xuU":
                n = {"x": 2, "u": 4, "U": 8}[e]
                h = self.src[self.i:self.i + n]
                self.i += n
                try:
                    return int(h, 16)
                except ValueError:
                    self.err(f"bad hex escape {h!r}")
            self.err(f"unknown escape \\{e}")
        self.i += 1
        return ord(ch)

    def parse(self):
        self.ws()
        while self.i < len(self.src):
            nm = self.name()
            self.ws(newlines=False)
            if not self.src.startswith("::=", self.i):
                self.err("expected ::=")
            self.i += 3
            rid = self.rule_id(nm)
            alts = self.alternatives(top=True)
            if self.rules[rid] is not None:
                self.err(f"rule {nm!r} defined twice")
            self.rules[rid] = alts
            self.ws()
        for nm, rid in self.names.items():
            if self.rules[rid] is None:
                raise GbnfError(f"undefined rule {nm!r}")
        if "root" not in self.names:
            raise GbnfError("grammar has no 'root' rule")
        return self.names["root"]

    def alternatives(self, top=False):
        alts = [self.sequence(top)]
        while True:
            self.ws(newlines=not top or self._continues())
            if self.i < len(self.src) and self.src[self.i] == "|":
                self.i += 1
                self.ws()
                alts.append(self.sequence(top))
            else:
                return alts

    def _continues(self) -> bool:
        # inside a top-level rule, a newline ends the rule unless the next line starts with '|'
        j = self.i
        while j < len(self.src) and self.src[j] in " \t\r\n":
            j += 1
        return j < len(self.src) and self.src[j] == "|"

    def sequence(self, top):
        seq = []
        while True:
            self.ws(newlines=not top)
            if self.i >= len(self.src):
                break
            ch = self.src[self.i]
            if ch == '"':
                self.i += 1
                lit = []
                while self.i < len(self.src) and self.src[self.i] != '"':
                    lit.append(self.char())
                if self.i >= len(self.src):
                    self.err("unterminated string")
                self.i += 1
                atoms = [CharSet(((c, c),)) for c in lit]
                elem = atoms if atoms else []
                seq.extend(self.quantify(elem, grouped=len(atoms) != 1))
            elif ch == "[":
                self.i += 1
                neg = False
                if self.i < len(self.src) and self.src[self.i] == "^":
                    neg = True
                    self.i += 1
                ranges = []
                while self.i < len(self.src) and self.src[self.i] != "]":
                    lo = self.char()
                    hi = lo
                    if self.src[self.i] == "-" and self.i + 1 < len(self.src) and self.src[self.i + 1] != "]":
                        self.i += 1
                        hi = self.char()
                    ranges.append((lo, hi))
                if self.i >= len(self.src):
                    self.err("unterminated character class")
                self.i += 1
                seq.extend(self.quantify([CharSet(tuple(ranges), neg)], grouped=False))
            elif ch == "(":
                self.i += 1
                self.ws()
                alts = self.alternatives()
                self.ws()
                if self.i >= len(self.src) or self.src[self.i] != ")":
                    self.err("expected )")
                self.i += 1
                rid = self.new_rule(alts)
                seq.extend(self.quantify([Ref(rid)], grouped=False))
            elif ch == ".":
                self.i += 1
                seq.extend(self.quantify([CharSet(((10, 10),), True)], grouped=False))
            elif ch.isalpha() or ch == "_":
                j = self.i
                nm = self.name()
                self.ws(newlines=False)
                if self.src.startswith("::=", self.i):  # next rule starts
                    self.i = j
                    break
                self.i = j
                nm = self.name()
                seq.extend(self.quantify([Ref(self.rule_id(nm))], grouped=False))
            else:
                break
        return seq

    def quantify(self, elems, grouped):
        if self.i >= len(self.src) or self.src[self.i] not in "*+?":
            return elems
        q = self.src[self.i]
        self.i += 1
        if grouped or len(elems) != 1:
            elems = [Ref(self.new_rule([list(elems)]))]
        x = elems[0]
        if q == "?":
            return [Ref(self.new_rule([[x], []]))]
        star = self.new_rule(None)
        self.rules[star] = [[x, Ref(star)], []]
        if q == "*":
            return [Ref(star)]
        return [x, Ref(star)]


class GbnfGrammar:
    def __init__(self, rules, root: int, names: dict[str, int]):
        self.rules = rules
        self.root = root
        self.names = names

    @classmethod
    def parse(cls, src: str) -> "GbnfGrammar":
        p = _Parser(src)
        root = p.parse()
        return cls(p.rules, root, dict(p.names))

    # stacks hold (rule, alt, pos) frames; the top frame's element is the next to match
    @functools.lru_cache(maxsize=65536)
    def expand(self, stack: tuple) -> frozenset:
        """Resolve the stack until its top is a character set (or the stack is empty)."""
        if not stack:
            return frozenset([()])
        rule, alt, pos = stack[-1]
        elems = self.rules[rule][alt]
        if pos >= len(elems):
            return self.expand(stack[:-1])
        e = elems[pos]
        if isinstance(e, CharSet):
            return frozenset([stack])
        rest = stack[:-1] + ((rule, alt, pos + 1),)
        out = set()
        for a in range(len(self.rules[e.rule])):
            out |= self.expand(rest + ((e.rule, a, 0),))
        return frozenset(out)

    def initial(self) -> frozenset:
        out = set()
        for a in range(len(self.rules[self.root])):
            out |= self.expand(((self.root, a, 0),))
        return frozenset(out)

    @functools.lru_cache(maxsize=262144)
    def advance(self, stacks: frozenset, c: int) -> frozenset:
        out = set()
        for st in stacks:
            if not st:
                continue
            rule, alt, pos = st[-1]
            e = self.rules[rule][alt][pos]
            if e.match(c):
                out |= self.expand(st[:-1] + ((rule, alt, pos + 1),))
        return frozenset(out)


class GbnfState:
    """Character-level recogniser state (reference ``GbnfState``)."""

    def __init__(self, grammar: GbnfGrammar):
        self.grammar = grammar
        self.stacks = grammar.initial()
        self._out: list[str] = []
        self.error = False

    def can_push_str(self, s: str) -> bool:
        st = self.stacks
        for ch in s:
            st = self.grammar.advance(st, ord(ch))
            if not st:
                return False
        return True

    def push_char(self, ch: str) -> bool:
        nxt = self.grammar.advance(self.stacks, ord(ch))
        if not nxt:
            self.error = True
            return False
        self.stacks = nxt
        self._out.append(ch)
        return True

    def is_complete(self) -> bool:
        return () in self.stacks

    def is_error(self) -> bool:
        return self.error

    def output(self) -> str:
        return "".join(self._out)


class _Trie:
    __slots__ = ("children", "ids")

    def __init__(self):
        self.children: dict[int, _Trie] = {}
        self.ids: list[int] = []


@functools.lru_cache(maxsize=8)
def _build_trie(token_texts: tuple) -> _Trie:
    root = _Trie()
    for i, t in enumerate(token_texts):
        node = root
        for ch in t:
            node = node.children.setdefault(ord(ch), _Trie())
        node.ids.append(i)
    return root


JSON_GBNF = r'''
root   ::= ws value ws
value  ::= object | array | string | number | ("true" | "false" | "null")
object ::= "{" ws ( string ws ":" ws value ( ws "," ws string ws ":" ws value )* )? ws "}"
array  ::= "[" ws ( value ( ws "," ws value )* )? ws "]"
string ::= "\"" ( [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] ) )* "\""
number ::= "-"? ( "0" | [1-9] [0-9]* ) ( "." [0-9]+ )? ( [eE] [-+]? [0-9]+ )?
ws     ::= [ \t\n]*
'''


class GbnfConstraint:
    """Grammar constraint over a vocabulary (reference ``GbnfConstraint``)."""

    def __init__(self, grammar: GbnfGrammar, token_texts: list[str], source: str = ""):
        self.grammar = grammar
        self.token_texts = tuple(token_texts)
        self.state = GbnfState(grammar)
        self.source = source
        self.eos_id: int | None = None

    # -- builders ----------------------------------------------------------
    @classmethod
    def from_str(cls, grammar_src: str, token_texts: list[str]) -> "GbnfConstraint":
        return cls(GbnfGrammar.parse(grammar_src), token_texts, grammar_src)

    @classmethod
    def json_mode(cls, token_texts: list[str]) -> "GbnfConstraint":
        return cls.from_str(JSON_GBNF, token_texts)

    @classmethod
    def identifier(cls, token_texts: list[str]) -> "GbnfConstraint":
        return cls.from_str("root ::= [a-zA-Z_] [a-zA-Z0-9_]*", token_texts)

    @classmethod
    def integer(cls, token_texts: list[str]) -> "GbnfConstraint":
        return cls.from_str('root ::= "-"? [0-9]+', token_texts)

    @classmethod
    def choice(cls, options: list[str], token_texts: list[str]) -> "GbnfConstraint":
        if not options:
            raise GbnfError("choice() requires at least one option")
        rhs = " | ".join('"' + o.replace("\\", "\\\\").replace('"', '\\"') + '"' for o in options)
        return cls.from_str(f"root ::= {rhs}", token_texts)

    # -- per-step API ------------------------------------------------------
    def step_mask(self) -> list[bool]:
        allowed = [False] * len(self.token_texts)
        g = self.grammar

        def walk(node: _Trie, stacks: frozenset):
            for i in node.ids:
                allowed[i] = True
            for c, child in node.children.items():
                nxt = g.advance(stacks, c)
                if nxt:
                    walk(child, nxt)

        root = _build_trie(self.token_texts)
        for c, child in root.children.items():
            nxt = g.advance(self.state.stacks, c)
            if nxt:
                walk(child, nxt)
        # empty-text tokens never advance the grammar: keep them masked
        if self.eos_id is not None and self.state.is_complete() and 0 <= self.eos_id < len(allowed):
            allowed[self.eos_id] = True
        return allowed

    def step_bitmask(self) -> torch.Tensor:
        """Allowed tokens packed 32 per int32 word (the device sampler's mask format)."""
        m = torch.tensor(self.step_mask(), dtype=torch.bool)
        V = m.numel()
        pad = (-V) % 32
        if pad:
            m = torch.cat([m, torch.zeros(pad, dtype=torch.bool)])
        bits = m.view(-1, 32).to(torch.int64) << torch.arange(32, dtype=torch.int64)
        words = bits.sum(-1)
        return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)

    def apply_to_logits(self, logits):
        mask = self.step_mask()
        if isinstance(logits, torch.Tensor):
            m = torch.tensor(mask, dtype=torch.bool, device=logits.device)
            logits.masked_fill_(~m[: logits.numel()], float("-inf"))
            return logits
        for i, ok in enumerate(mask):
            if not ok:
                logits[i] = float("-inf")
        return logits

    def can_push_token(self, text: str) -> bool:
        return self.state.can_push_str(text)

    def push_token(self, decoded) -> None:
        if isinstance(decoded, int):
            decoded = self.token_texts[decoded] if 0 <= decoded < len(self.token_texts) else ""
        for ch in decoded:
            if not self.state.push_char(ch):
                break

    def validate_path(self, tokens: list[int], tokenizer=None) -> bool:
        st = GbnfState(self.grammar)
        st.stacks = self.state.stacks
        for t in tokens:
            text = tokenizer.decode_token(t) if tokenizer is not None else self.token_texts[t]
            if not st.can_push_str(text):
                return False
            for ch in text:
                st.push_char(ch)
        return True

    def is_complete(self) -> bool:
        return self.state.is_complete()

    def output(self) -> str:
        return self.state.output()

    def reset(self):
        self.state = GbnfState(self.grammar)

    def clone(self) -> "GbnfConstraint":
        c = GbnfConstraint(self.grammar, list(self.token_texts), self.source)
        c.state.stacks = self.state.stacks
        c.state._out = list(self.state._out)
        c.eos_id = self.eos_id
        return c
