"""Ghost drafting policy (reference ``src/ghost_drafting.rs``: ghost model selection by free
memory, platform time-to-first-token profiles, feasibility against first-layer I/O time,
AcceptanceTracker with an EMA acceptance rate and adaptive draft length, GhostSession,
SpeculativeCheckpointTree).

On B200 the "ghost" is a small draft model held in HBM next to the target (the reference
keeps it in host RAM while the target streams from disk); selection is by free device memory,
and ``AcceptanceTracker`` drives the draft depth of ``SpeculativeDecoder(adaptive=True)``
from measured acceptances. A rollback here is a block-table truncation, so the checkpoint tree
only records the token diffs of a draft branch.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

DEFAULT_DRAFT_K = 4
DEFAULT_ACCEPTANCE_RATE = 0.75


class GhostModel(str, enum.Enum):
    LLAMA32_3B = "llama3.2-3b"
    LLAMA32_1B = "llama3.2-1b"

    @property
    def size_mb(self) -> float:
        return {GhostModel.LLAMA32_3B: 1900.0, GhostModel.LLAMA32_1B: 700.0}[self]

    @property
    def params_b(self) -> float:
        return {GhostModel.LLAMA32_3B: 3.0, GhostModel.LLAMA32_1B: 1.0}[self]

    @property
    def display_name(self) -> str:
        return {GhostModel.LLAMA32_3B: "Llama 3.2 3B Q4_K_M", GhostModel.LLAMA32_1B: "Llama 3.2 1B Q4_K_M"}[self]

    def __str__(self) -> str:
        return f"{self.display_name} ({self.size_mb / 1024:.1f} GB)"


def select_ghost_model(available_mb: float) -> GhostModel | None:
    """>= 4000 MB free: the 3B drafter; >= 2000 MB: the 1B drafter; else none."""
    if available_mb >= 4000:
        return GhostModel.LLAMA32_3B
    if available_mb >= 2000:
        return GhostModel.LLAMA32_1B
    return None


@dataclass
class GhostPlatformProfile:
    name: str
    ttft_ms: float
    model: GhostModel
    method: str
    cpu_only: bool = False

    @classmethod
    def b200(cls) -> "GhostPlatformProfile":
        # a 1B Q4_K drafter decodes in well under a millisecond per token on one B200
        return cls("NVIDIA B200 (HBM-resident drafter)", 5.0, GhostModel.LLAMA32_1B, "CUDA graph decode")

    @classmethod
    def nvidia_gpu(cls) -> "GhostPlatformProfile":
        return cls("NVIDIA GPU", 80.0, GhostModel.LLAMA32_3B, "CUDA")

    @classmethod
    def cpu(cls, name: str = "CPU", ttft_ms: float = 400.0) -> "GhostPlatformProfile":
        return cls(name, ttft_ms, GhostModel.LLAMA32_1B, "CPU", cpu_only=True)

    @classmethod
    def custom(cls, name: str, ttft_ms: float, model: GhostModel, method: str, cpu_only: bool):
        return cls(name, ttft_ms, model, method, cpu_only)


@dataclass
class FeasibilityResult:
    storage_name: str
    t_io_first_layer_ms: float
    ghost_ttft_ms: float
    speedup: float
    feasible: bool
    applicable: bool


def check_feasibility(t_io_first_layer_ms: float, profile: GhostPlatformProfile,
                      main_model_cpu_only: bool) -> FeasibilityResult:
    """Useful iff the drafter answers before the target's first layer arrives; not applicable
    when the target itself runs on the CPU (no separate device to draft on)."""
    applicable = not main_model_cpu_only
    speedup = t_io_first_layer_ms / profile.ttft_ms if profile.ttft_ms > 0 else float("inf")
    return FeasibilityResult("", t_io_first_layer_ms, profile.ttft_ms, speedup,
                             applicable and profile.ttft_ms < t_io_first_layer_ms, applicable)


def feasibility_matrix(profile: GhostPlatformProfile, layer_size_mb: float,
                       storages: list[tuple[str, float]] | None = None) -> list[FeasibilityResult]:
    """Feasibility per storage tier (name, MB/s) for one layer of ``layer_size_mb``."""
    storages = storages or [("USB 3.0 HDD", 80.0), ("5400 RPM HDD", 110.0), ("7200 RPM HDD", 160.0),
                            ("SATA SSD", 500.0), ("NVMe Gen5", 12000.0), ("pinned host -> HBM", 50000.0)]
    out = []
    for name, mbps in storages:
        r = check_feasibility(layer_size_mb / mbps * 1000.0, profile, False)
        r.storage_name = name
        out.append(r)
    return out


@dataclass
class AcceptanceTracker:
    draft_k: int = DEFAULT_DRAFT_K
    ema_rate: float = DEFAULT_ACCEPTANCE_RATE
    ema_alpha: float = 0.2
    total_drafted: int = 0
    total_accepted: int = 0
    rejection_streak: int = 0
    history: list = field(default_factory=list)

    def report_batch(self, drafted: int, accepted: int):
        accepted = min(accepted, drafted)
        self.total_drafted += drafted
        self.total_accepted += accepted
        self.history.append((drafted, accepted))
        rate = accepted / drafted if drafted > 0 else 0.0
        self.ema_rate = self.ema_alpha * rate + (1 - self.ema_alpha) * self.ema_rate
        self.rejection_streak = self.rejection_streak + 1 if accepted == 0 else 0

    def acceptance_rate(self) -> float:
        return self.total_accepted / self.total_drafted if self.total_drafted else DEFAULT_ACCEPTANCE_RATE

    def effective_tokens(self) -> float:
        return self.ema_rate * self.draft_k

    def ghost_accept_time_ms(self, t_token_ms: float) -> float:
        return self.ema_rate * self.draft_k * t_token_ms

    def net_ghost_contribution_ms(self, t_token_ms: float) -> float:
        return self.ghost_accept_time_ms(t_token_ms) * 0.75

    def batch_count(self) -> int:
        return len(self.history)

    def should_disable(self) -> bool:
        """Five fully rejected batches in a row."""
        return self.rejection_streak >= 5

    def suggest_k(self, k_max: int = 8) -> int:
        """High acceptance lengthens the draft, low acceptance shortens it."""
        if self.ema_rate >= 0.85:
            return min(self.draft_k + 2, k_max)
        if self.ema_rate >= 0.60:
            return self.draft_k
        if self.ema_rate >= 0.30:
            return max(1, self.draft_k - 1)
        return 1

    def __str__(self) -> str:
        return (f"Ghost: a={self.acceptance_rate() * 100:.1f}% (EMA={self.ema_rate * 100:.1f}%), "
                f"k={self.draft_k}, {self.total_accepted}/{self.total_drafted} accepted, {len(self.history)} batches")


@dataclass
class GhostSession:
    model: GhostModel | None
    platform: GhostPlatformProfile
    t_io_first_layer_ms: float
    main_model_cpu_only: bool
    available_mb: float
    tracker: AcceptanceTracker = field(default_factory=AcceptanceTracker)
    active: bool = False

    @classmethod
    def create(cls, available_mb: float, platform: GhostPlatformProfile, t_io_first_layer_ms: float,
               main_model_cpu_only: bool = False) -> "GhostSession":
        model = select_ghost_model(available_mb)
        feas = check_feasibility(t_io_first_layer_ms, platform, main_model_cpu_only)
        return cls(model, platform, t_io_first_layer_ms, main_model_cpu_only, available_mb,
                   active=model is not None and feas.feasible)

    def report_verification(self, drafted: int, accepted: int):
        self.tracker.report_batch(drafted, accepted)
        if self.tracker.should_disable():
            self.active = False

    def perceived_ttft_ms(self) -> float:
        return 5.0 + self.platform.ttft_ms if self.active else self.t_io_first_layer_ms

    def ttft_speedup(self) -> float:
        if self.active and self.platform.ttft_ms > 0:
            return self.t_io_first_layer_ms / self.perceived_ttft_ms()
        return 1.0

    def rho_contribution(self, t_token_ms: float) -> float:
        return self.tracker.net_ghost_contribution_ms(t_token_ms) if self.active else 0.0


@dataclass
class SpeculativeCheckpointTree:
    """Token diffs of a draft branch relative to its root position; rolling back is a
    truncation of the sequence to ``root_pos`` plus these diffs, no KV copy."""
    root_pos: int
    token_diffs: list = field(default_factory=list)

    def push_diff(self, offset: int, token_id: int):
        self.token_diffs.append((offset, token_id))

    def tokens_after(self, base: list[int]) -> list[int]:
        out = list(base[: self.root_pos])
        for off, tok in sorted(self.token_diffs):
            pos = self.root_pos + off
            if pos < len(out):
                out[pos] = tok
            else:
                out.extend([0] * (pos - len(out)))
                out.append(tok)
        return out

    def rollback(self, n_accepted: int) -> int:
        """Keep the first ``n_accepted`` diffs; returns the sequence length to truncate to."""
        self.token_diffs = sorted(self.token_diffs)[:n_accepted]
        return self.root_pos + n_accepted
