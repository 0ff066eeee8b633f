"""Per-sample accounting of the model-local PISA override (host-side, no
tensor data retained).  Same contract as the reference's
rdna35_block_attention/pisa_runtime.py:12-153: counters of hits per layer,
fallback reasons, shapes, backends and hit contexts under a lock, and
``verify`` that every expected layer ran once per forward."""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass, field
from threading import Lock
from typing import Iterable

PISA_RUNTIME_ATTACHMENT = "rdna35_pisa_runtime_state"


def _fmt(counter: Counter) -> str:
    return ",".join(f"{key}:{count}" for key, count in sorted(counter.items())) or "-"


@dataclass
class PISARuntimeState:
    armed: bool = False
    executed: bool = False
    verified: bool = False
    failed: bool = False
    per_layer_hits: Counter = field(default_factory=Counter)
    fallback_reasons: Counter = field(default_factory=Counter)
    self_calls: int = 0
    cross_calls: int = 0
    shape_counts: Counter = field(default_factory=Counter)
    backend_counts: Counter = field(default_factory=Counter)
    hit_context_counts: Counter = field(default_factory=Counter)
    first_error: str | None = None
    quality_sample: str | None = None
    validated_profiles: set = field(default_factory=set)
    expected_layers: tuple = ()
    _expected: int | None = field(default=None, init=False, repr=False)
    _lock: Lock = field(default_factory=Lock, init=False, repr=False)

    @staticmethod
    def expected_calls(actual_forwards: int, start_layer: int = 20, total_layers: int = 28,
                       layers: Iterable[int] | None = None) -> int:
        if actual_forwards < 0:
            raise ValueError("actual_forwards must be non-negative")
        if start_layer < 0 or total_layers < start_layer:
            raise ValueError("expected 0 <= start_layer <= total_layers")
        chosen = tuple(range(start_layer, total_layers)) if layers is None else tuple(layers)
        return actual_forwards * len(chosen)

    def reset(self, *, armed: bool | None = None) -> None:
        with self._lock:
            if armed is not None:
                self.armed = armed
            self.executed = self.verified = self.failed = False
            for counter in (self.per_layer_hits, self.fallback_reasons, self.shape_counts, self.backend_counts,
                            self.hit_context_counts):
                counter.clear()
            self.self_calls = self.cross_calls = 0
            self.first_error = None
            self.quality_sample = None
            self.validated_profiles.clear()
            self._expected = None

    def record(self, *, layer: int | None = None, is_self_attention: bool | None = None,
               shape: Iterable[int] | None = None, fallback_reason: str | None = None,
               error: BaseException | str | None = None, backend: str | None = None, context: str | None = None,
               quality: str | None = None) -> None:
        with self._lock:
            if is_self_attention is True:
                self.self_calls += 1
            elif is_self_attention is False:
                self.cross_calls += 1
            if shape is not None:
                self.shape_counts[tuple(int(x) for x in shape)] += 1
            if fallback_reason is not None:
                self.fallback_reasons[str(fallback_reason)] += 1
            if error is not None:
                self.failed = True
                if self.first_error is None:
                    self.first_error = str(error)
            if backend is not None:
                self.backend_counts[str(backend)] += 1
                if context is not None:
                    self.hit_context_counts[str(context)] += 1
            if quality is not None and self.quality_sample is None:
                self.quality_sample = str(quality)
            if layer is not None:
                self.executed = True
                self.per_layer_hits[int(layer)] += 1

    def verify(self, actual_forwards: int, start_layer: int = 20, total_layers: int = 28) -> bool:
        layers = self.expected_layers or tuple(range(start_layer, total_layers))
        expected = self.expected_calls(actual_forwards, layers=layers)
        with self._lock:
            self._expected = expected
            if self.failed:
                self.verified = False
                return False
            unexpected = sorted(set(self.per_layer_hits).difference(layers))
            missing = [layer for layer in layers if self.per_layer_hits[layer] != actual_forwards]
            actual = sum(self.per_layer_hits.values())
            if unexpected or missing or actual != expected:
                self.failed = True
                self.verified = False
                if self.first_error is None:
                    self.first_error = f"PISA hits={actual}, expected={expected}"
                return False
            self.verified = True
            return True

    def is_profile_validated(self, profile: tuple) -> bool:
        with self._lock:
            return profile in self.validated_profiles

    def mark_profile_validated(self, profile: tuple) -> None:
        with self._lock:
            self.validated_profiles.add(profile)

    def report(self) -> str:
        with self._lock:
            hits = sum(self.per_layer_hits.values())
            expected = "?" if self._expected is None else str(self._expected)
            shapes = ",".join(f"{s}:{c}" for s, c in sorted(self.shape_counts.items())) or "-"
            return (
                f"PISA armed={int(self.armed)} executed={int(self.executed)} verified={int(self.verified)} "
                f"failed={int(self.failed)} hits={hits}/{expected} self={self.self_calls} cross={self.cross_calls} "
                f"fallbacks={_fmt(self.fallback_reasons)} backends={_fmt(self.backend_counts)} "
                f"hit_contexts={_fmt(self.hit_context_counts)} shapes={shapes} "
                f"quality={self.quality_sample or '-'} first_error={self.first_error or '-'}"
            )
