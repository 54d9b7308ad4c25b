"""String helpers that need no engine (reference ``python/air_rs/utils.py``)."""
from __future__ import annotations

from ..structured.chat_template import ChatFormat, ChatTemplate

_SUPPORTED = ("chatml", "gemma", "llama3", "mistral", "phi3")


def format_chat(messages: list[dict[str, str]], template: str = "chatml", *,
                add_generation_prompt: bool = True) -> str:
    """Render a conversation in a model family's prompt format."""
    key = template.lower()
    if key not in _SUPPORTED:
        raise ValueError(f"Unknown template {template!r}. Supported: {', '.join(_SUPPORTED)}")
    return ChatTemplate(ChatFormat(key), add_generation_prompt).apply(messages)


def count_tokens_approx(text: str) -> int:
    """Rough token count (characters / 4, at least 1), no tokenizer needed."""
    return max(1, len(text) // 4)
