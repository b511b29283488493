"""Per-chunk latency bookkeeping, with the reference's `Timing` interface
(`src/so101_smolvla_edge/model/timing.py:11-38`): last_ms, history, add, summary."""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class Timing:
    last_ms: float = 0.0
    history: list[float] = field(default_factory=list)

    def add(self, ms: float) -> None:
        """Record one chunk; past 1000 entries the oldest 500 are dropped."""
        self.last_ms = ms
        self.history.append(ms)
        if len(self.history) > 1000:
            del self.history[:500]

    def summary(self) -> dict:
        """n, p50/p90/p99 and max of the recorded latencies in ms ({} when empty)."""
        h = sorted(self.history)
        if not h:
            return {}

        def q(p: float) -> float:
            return h[min(len(h) - 1, int(p * (len(h) - 1)))]

        return {"n": len(h), "p50_ms": q(0.5), "p90_ms": q(0.9), "p99_ms": q(0.99), "max_ms": h[-1]}
