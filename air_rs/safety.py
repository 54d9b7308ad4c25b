"""Content safety gate (reference ``src/content_safety.rs``): a keyword classifier with harm
categories, a policy (threshold, block / warn / pass, which sides to screen) and a gate the
REST server consults before generating and before returning text.

The term lists are this project's own, short and configurable (``extra_terms``); a deployment
that needs a real classifier plugs one in through the same ``classify(text) -> SafetyVerdict``
interface.
"""
from __future__ import annotations

import enum
import re
from dataclasses import dataclass


class HarmCategory(str, enum.Enum):
    NSFW = "nsfw"
    TOXIC = "toxic"
    VIOLENCE = "violence"
    SELF_HARM = "self_harm"
    ILLEGAL = "illegal"


@dataclass
class SafetyVerdict:
    safe: bool
    category: HarmCategory | None = None
    confidence: float = 0.0
    reason: str | None = None

    @classmethod
    def ok(cls) -> "SafetyVerdict":
        return cls(True)

    @classmethod
    def blocked(cls, category: HarmCategory, confidence: float, reason: str) -> "SafetyVerdict":
        return cls(False, category, confidence, reason)


# checked in this order; first match wins
DEFAULT_TERMS: dict[HarmCategory, tuple[str, ...]] = {
    HarmCategory.ILLEGAL: ("synthesize methamphetamine", "make a pipe bomb", "counterfeit currency",
                           "launder money"),
    HarmCategory.VIOLENCE: ("how to kill someone", "mass shooting plan", "torture a person"),
    HarmCategory.SELF_HARM: ("how to commit suicide", "ways to self-harm", "kill myself"),
    HarmCategory.NSFW: ("explicit sexual content", "pornographic"),
    HarmCategory.TOXIC: ("subhuman vermin", "go die in a fire"),
}


class KeywordClassifier:
    def __init__(self, extra_terms: dict[HarmCategory, list[str]] | None = None, confidence: float = 0.90):
        self.terms = {c: list(t) for c, t in DEFAULT_TERMS.items()}
        for c, ts in (extra_terms or {}).items():
            self.terms.setdefault(HarmCategory(c), []).extend(t.lower() for t in ts)
        self.confidence = confidence

    def classify(self, text: str) -> SafetyVerdict:
        if not text:
            return SafetyVerdict.ok()
        low = re.sub(r"\s+", " ", text.lower())
        for cat, terms in self.terms.items():
            for t in terms:
                if t in low:
                    return SafetyVerdict.blocked(cat, self.confidence, f"keyword match: '{t}'")
        return SafetyVerdict.ok()


class SafetyAction(str, enum.Enum):
    BLOCK = "block"
    WARN = "warn"
    PASS = "pass"


@dataclass
class SafetyPolicy:
    threshold: float = 0.80
    action: SafetyAction = SafetyAction.BLOCK
    screen_input: bool = True
    screen_output: bool = True


class ContentSafetyGate:
    def __init__(self, classifier=None, policy: SafetyPolicy | None = None):
        self.classifier = classifier or KeywordClassifier()
        self.policy = policy or SafetyPolicy()
        self.blocked = 0
        self.warned = 0

    def check(self, text: str) -> SafetyVerdict:
        v = self.classifier.classify(text)
        return v if (not v.safe and v.confidence >= self.policy.threshold) else SafetyVerdict.ok()

    def should_block(self, text: str) -> bool:
        v = self.check(text)
        if v.safe:
            return False
        if self.policy.action == SafetyAction.BLOCK:
            self.blocked += 1
            return True
        if self.policy.action == SafetyAction.WARN:
            self.warned += 1
        return False

    @staticmethod
    def block_reason(v: SafetyVerdict) -> str:
        return f"content_policy_violation:{v.category.value}" if v.category else "content_policy_violation"
