"""Modelfile (reference ``src/modelfile.rs``): FROM / SYSTEM / TEMPLATE / STOP / PARAMETER
lines (comments with ``#``, values optionally quoted, triple-quoted multi-line values) that
set a model's default system prompt and sampling parameters.
"""
from __future__ import annotations

from dataclasses import dataclass, field


def _unquote(s: str) -> str:
    s = s.strip()
    for q in ('"""', '"', "'"):
        if len(s) >= 2 * len(q) and s.startswith(q) and s.endswith(q):
            return s[len(q):-len(q)]
    return s


@dataclass
class Modelfile:
    from_: str | None = None
    system: str | None = None
    template: str | None = None
    stop: list[str] = field(default_factory=list)
    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    repetition_penalty: float | None = None
    max_tokens: int | None = None

    @classmethod
    def parse(cls, text: str) -> "Modelfile":
        mf = cls()
        lines = text.splitlines()
        i = 0
        while i < len(lines):
            line = lines[i].strip()
            i += 1
            if not line or line.startswith("#"):
                continue
            cmd, _, rest = line.partition(" ")
            cmd, rest = cmd.upper(), rest.strip()
            if rest.startswith('"""') and not (len(rest) >= 6 and rest.endswith('"""')):
                buf = [rest[3:]]
                while i < len(lines) and not lines[i].rstrip().endswith('"""'):
                    buf.append(lines[i])
                    i += 1
                if i < len(lines):
                    buf.append(lines[i].rstrip()[:-3])
                    i += 1
                rest = '"""' + "\n".join(buf) + '"""'
            val = _unquote(rest)
            if cmd == "FROM":
                mf.from_ = val
            elif cmd == "SYSTEM":
                mf.system = val
            elif cmd == "TEMPLATE":
                mf.template = val
            elif cmd == "STOP" and val:
                mf.stop.append(val)
            elif cmd == "PARAMETER":
                name, _, pv = rest.partition(" ")
                name, pv = name.lower(), pv.strip()
                try:
                    if name == "temperature":
                        mf.temperature = float(pv)
                    elif name == "top_p":
                        mf.top_p = float(pv)
                    elif name == "top_k":
                        mf.top_k = int(pv)
                    elif name in ("repeat_penalty", "repetition_penalty"):
                        mf.repetition_penalty = float(pv)
                    elif name in ("max_tokens", "num_predict"):
                        mf.max_tokens = int(pv)
                    elif name == "stop" and _unquote(pv):
                        mf.stop.append(_unquote(pv))
                except ValueError:
                    pass
        return mf

    @classmethod
    def load(cls, path: str) -> "Modelfile":
        with open(path) as f:
            return cls.parse(f.read())

    def apply_to(self, cfg):
        """Fill a ``GenerateConfig`` (serve.dispatcher or api): system prompt and defaults."""
        if self.system:
            if not cfg.prompt:
                cfg.prompt = self.system
            elif self.system not in cfg.prompt:
                cfg.prompt = f"System: {self.system}\n\nUser: {cfg.prompt}"
        for k in ("temperature", "top_p", "top_k", "repetition_penalty", "max_tokens"):
            v = getattr(self, k)
            if v is not None and hasattr(cfg, k):
                setattr(cfg, k, v)
        if self.stop and hasattr(cfg, "stop"):
            cfg.stop = list(dict.fromkeys(list(cfg.stop or []) + self.stop))
        return cfg
