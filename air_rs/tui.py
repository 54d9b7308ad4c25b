"""Terminal front-end helpers (reference ``src/tui.rs``): status bar, streaming display,
generation stats and an interactive REPL (the reference ships these unwired)."""
from __future__ import annotations

import shutil
import sys
import time
from dataclasses import dataclass


@dataclass
class GenerationStats:
    tokens: int = 0
    elapsed_s: float = 0.0
    ttft_ms: float = 0.0

    @property
    def tokens_per_second(self) -> float:
        return self.tokens / self.elapsed_s if self.elapsed_s > 0 else 0.0


class StatusBar:
    def __init__(self, model: str, stream=sys.stderr):
        self.model, self.stream = model, stream

    def render(self, stats: GenerationStats) -> str:
        width = shutil.get_terminal_size((100, 20)).columns
        s = (f" {self.model} | {stats.tokens} tok | {stats.tokens_per_second:.1f} tok/s | "
             f"TTFT {stats.ttft_ms:.0f} ms ")
        return s[:width].ljust(min(width, len(s)))

    def show(self, stats: GenerationStats):
        self.stream.write("\r" + self.render(stats))
        self.stream.flush()


class StreamDisplay:
    def __init__(self, out=sys.stdout):
        self.out = out
        self.stats = GenerationStats()
        self._t0 = None

    def push(self, text: str):
        now = time.perf_counter()
        if self._t0 is None:
            self._t0 = now
        self.stats.tokens += 1
        self.stats.elapsed_s = now - self._t0
        self.out.write(text)
        self.out.flush()


def read_user_input(prompt: str = ">>> ", inp=input) -> str | None:
    try:
        line = inp(prompt)
    except EOFError:
        return None
    return None if line.strip() in ("/exit", "/quit") else line


def repl(model_path: str, inp=input, out=sys.stdout) -> int:
    """Multi-turn chat loop over ``Engine`` with the model family's chat template."""
    from .api import Engine, GenerateConfig
    from .structured.chat_template import ChatTemplate, detect_format
    eng = Engine.from_gguf(model_path)
    tmpl = ChatTemplate(detect_format(model_path, eng.core.tokenizer and {}))
    history = []
    while True:
        line = read_user_input(inp=inp)
        if line is None:
            return 0
        history.append({"role": "user", "content": line})
        disp = StreamDisplay(out)
        text = []
        ch = eng._stream_channel(tmpl.apply(history), GenerateConfig(max_tokens=512))
        for tok in ch:
            disp.push(tok)
            text.append(tok)
        out.write("\n")
        history.append({"role": "assistant", "content": "".join(text)})
