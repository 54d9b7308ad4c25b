"""Chat prompt formats (reference ``src/chat_template.rs`` and ``python/air_rs/utils.py``).

The token layouts are the published conversation formats of each model family (ChatML,
Llama-3, Mistral [INST], Phi-3, Gemma); they have to be reproduced exactly for the models
to behave, so the strings below are those formats, written out by us.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass


class Role(str, enum.Enum):
    SYSTEM = "system"
    USER = "user"
    ASSISTANT = "assistant"
    TOOL = "tool"

    @classmethod
    def parse(cls, s: str) -> "Role | None":
        try:
            return cls(s.lower())
        except ValueError:
            return None


@dataclass
class ChatMessage:
    role: str
    content: str

    @classmethod
    def system(cls, c):
        return cls("system", c)

    @classmethod
    def user(cls, c):
        return cls("user", c)

    @classmethod
    def assistant(cls, c):
        return cls("assistant", c)


class ChatFormat(str, enum.Enum):
    CHATML = "chatml"
    LLAMA3 = "llama3"
    MISTRAL = "mistral"
    PHI3 = "phi3"
    GEMMA = "gemma"
    RAW = "raw"


class ChatTemplate:
    def __init__(self, fmt: ChatFormat | str = ChatFormat.CHATML, add_generation_prompt: bool = True):
        self.format = ChatFormat(fmt)
        self.add_generation_prompt = add_generation_prompt

    def apply(self, messages) -> str:
        msgs = [m if isinstance(m, ChatMessage) else ChatMessage(m["role"], m.get("content") or "")
                for m in messages]
        return getattr(self, "_" + self.format.value)(msgs)

    def _chatml(self, msgs):
        out = "".join(f"<|im_start|>{m.role}\n{m.content}<|im_end|>\n" for m in msgs)
        return out + ("<|im_start|>assistant\n" if self.add_generation_prompt else "")

    def _llama3(self, msgs):
        out = "<|begin_of_text|>"
        for m in msgs:
            out += f"<|start_header_id|>{m.role}<|end_header_id|>\n\n{m.content}<|eot_id|>"
        return out + ("<|start_header_id|>assistant<|end_header_id|>\n\n" if self.add_generation_prompt else "")

    def _mistral(self, msgs):
        out, system = "<s>", ""
        for m in msgs:
            if m.role == "system":
                system = m.content + "\n\n"
            elif m.role == "user":
                out += f"[INST] {system}{m.content} [/INST]"
                system = ""
            else:
                out += f" {m.content}</s>"
        return out

    def _phi3(self, msgs):
        out = "".join(f"<|{m.role}|>\n{m.content}<|end|>\n" for m in msgs)
        return out + ("<|assistant|>\n" if self.add_generation_prompt else "")

    def _gemma(self, msgs):
        out, system = "<bos>", ""
        for m in msgs:
            if m.role == "system":
                system = m.content + "\n\n"
                continue
            role = "model" if m.role == "assistant" else "user"
            content = (system + m.content) if role == "user" else m.content
            system = "" if role == "user" else system
            out += f"<start_of_turn>{role}\n{content}<end_of_turn>\n"
        return out + ("<start_of_turn>model\n" if self.add_generation_prompt else "")

    def _raw(self, msgs):
        return "\n".join(m.content for m in msgs)


def detect_format(model_name: str = "", metadata: dict | None = None) -> ChatFormat:
    md = metadata or {}
    tmpl = str(md.get("tokenizer.chat_template", ""))
    arch = str(md.get("general.architecture", "")).lower()
    name = (model_name or str(md.get("general.name", ""))).lower()
    if "<|im_start|>" in tmpl or "qwen" in name or "qwen" in arch:
        return ChatFormat.CHATML
    if "<|start_header_id|>" in tmpl or "llama-3" in name or "llama3" in name:
        return ChatFormat.LLAMA3
    if "[INST]" in tmpl or "mistral" in name or "mixtral" in name or arch == "mistral":
        return ChatFormat.MISTRAL
    if "<|end|>" in tmpl or "phi-3" in name or "phi3" in name or arch == "phi3":
        return ChatFormat.PHI3
    if "<start_of_turn>" in tmpl or "gemma" in name or arch.startswith("gemma"):
        return ChatFormat.GEMMA
    if arch == "llama":
        return ChatFormat.LLAMA3
    return ChatFormat.CHATML
