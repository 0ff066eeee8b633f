"""Per-sample accounting of the model-local PISA override.

Contract (the public surface of the reference's
rdna35_block_attention/pisa_runtime.py:12-153, which other modules, the
report node and user code read): a ``PISARuntimeState`` object exposing the
flags ``armed / executed / verified / failed``, the tallies
``per_layer_hits / fallback_reasons / shape_counts / backend_counts /
hit_context_counts`` (``collections.Counter``), the call counts
``self_calls / cross_calls``, ``first_error``, ``quality_sample``,
``validated_profiles`` and ``expected_layers``; the operations
``expected_calls``, ``reset``, ``record``, ``verify``,
``is_profile_validated``, ``mark_profile_validated`` and the one-line
``report``.  No tensor data is retained.  All mutation happens under one
lock because ComfyUI may run attention from several threads.

This implementation keeps the tallies in a name -> Counter table so that
reset and report walk one list, and ``record`` treats each keyword as an
independent event.
"""
from __future__ import annotations

from collections import Counter
from threading import Lock
from typing import Iterable

PISA_RUNTIME_ATTACHMENT = "rdna35_pisa_runtime_state"

# report key -> tally attribute, in report order
_REPORTED_TALLIES = (("fallbacks", "fallback_reasons"), ("backends", "backend_counts"),
                     ("hit_contexts", "hit_context_counts"))
_ALL_TALLIES = ("per_layer_hits", "fallback_reasons", "shape_counts", "backend_counts", "hit_context_counts")


def _layers(start_layer: int, total_layers: int, layers: Iterable[int] | None) -> tuple[int, ...]:
    if start_layer < 0 or total_layers < start_layer:
        raise ValueError("expected 0 <= start_layer <= total_layers")
    return tuple(range(start_layer, total_layers)) if layers is None else tuple(layers)


def _render(tally: Counter) -> str:
    """'key:count' pairs in key order, '-' when empty."""
    if not tally:
        return "-"
    return ",".join(f"{key}:{tally[key]}" for key in sorted(tally))


class PISARuntimeState:
    """Hit / fallback accounting of one sampling run of a patched model."""

    def __init__(self, armed: bool = False, executed: bool = False, verified: bool = False, failed: bool = False,
                 expected_layers: tuple = (), **tallies):
        unknown = set(tallies) - set(_ALL_TALLIES)
        if unknown:
            raise TypeError(f"unexpected arguments: {sorted(unknown)}")
        self.armed, self.executed, self.verified, self.failed = armed, executed, verified, failed
        for name in _ALL_TALLIES:
            setattr(self, name, Counter(tallies.get(name, ())))
        self.self_calls = 0
        self.cross_calls = 0
        self.first_error: str | None = None
        self.quality_sample: str | None = None
        self.validated_profiles: set = set()
        self.expected_layers = tuple(expected_layers)
        self._expected: int | None = None
        self._lock = Lock()

    def __repr__(self) -> str:
        return f"PISARuntimeState({self.report()})"

    @staticmethod
    def expected_calls(actual_forwards: int, start_layer: int = 20, total_layers: int = 28,
                       layers: Iterable[int] | None = None) -> int:
        """Override invocations a run of `actual_forwards` model forwards
        should produce: one per patched layer per forward."""
        if actual_forwards < 0:
            raise ValueError("actual_forwards must be non-negative")
        return actual_forwards * len(_layers(start_layer, total_layers, layers))

    def reset(self, *, armed: bool | None = None) -> None:
        with self._lock:
            if armed is not None:
                self.armed = armed
            self.executed = self.verified = self.failed = False
            for name in _ALL_TALLIES:
                getattr(self, name).clear()
            self.self_calls = self.cross_calls = 0
            self.first_error = self.quality_sample = None
            self.validated_profiles.clear()
            self._expected = None

    def record(self, *, layer: int | None = None, is_self_attention: bool | None = None,
               shape: Iterable[int] | None = None, fallback_reason: str | None = None,
               error: BaseException | str | None = None, backend: str | None = None, context: str | None = None,
               quality: str | None = None) -> None:
        """Count one override event; every keyword left None is ignored.
        A hit context is counted only together with the backend that ran."""
        with self._lock:
            if is_self_attention is not None:
                if is_self_attention:
                    self.self_calls += 1
                else:
                    self.cross_calls += 1
            if shape is not None:
                self.shape_counts[tuple(map(int, shape))] += 1
            if fallback_reason is not None:
                self.fallback_reasons[str(fallback_reason)] += 1
            if error is not None:
                self.failed = True
                self.first_error = self.first_error or str(error)
            if backend is not None:
                self.backend_counts[str(backend)] += 1
                if context is not None:
                    self.hit_context_counts[str(context)] += 1
            if quality is not None and self.quality_sample is None:
                self.quality_sample = str(quality)
            if layer is not None:
                self.per_layer_hits[int(layer)] += 1
                self.executed = True

    def _mismatch(self, layers: tuple[int, ...], actual_forwards: int, expected: int) -> str | None:
        hits = self.per_layer_hits
        total = sum(hits.values())
        stray = any(layer not in layers for layer in hits)
        uneven = any(hits[layer] != actual_forwards for layer in layers)
        if stray or uneven or total != expected:
            return f"PISA hits={total}, expected={expected}"
        return None

    def verify(self, actual_forwards: int, start_layer: int = 20, total_layers: int = 28) -> bool:
        """True when every expected layer ran exactly once per forward, no
        other layer ran and no error was recorded; otherwise marks the
        state failed (keeping the first error message)."""
        layers = self.expected_layers or _layers(start_layer, total_layers, None)
        expected = self.expected_calls(actual_forwards, layers=layers)
        with self._lock:
            self._expected = expected
            problem = None if self.failed else self._mismatch(layers, actual_forwards, expected)
            if self.failed or problem is not None:
                self.failed = True
                self.verified = False
                self.first_error = self.first_error or problem
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
        """One line: flags, hits/expected, call counts, tallies, quality
        sample and first error ('-' for anything empty)."""
        with self._lock:
            parts = [f"PISA armed={int(self.armed)}", f"executed={int(self.executed)}",
                     f"verified={int(self.verified)}", f"failed={int(self.failed)}",
                     f"hits={sum(self.per_layer_hits.values())}/{'?' if self._expected is None else self._expected}",
                     f"self={self.self_calls}", f"cross={self.cross_calls}"]
            parts += [f"{key}={_render(getattr(self, name))}" for key, name in _REPORTED_TALLIES]
            parts.append(f"shapes={_render(self.shape_counts)}")
            parts.append(f"quality={self.quality_sample or '-'}")
            parts.append(f"first_error={self.first_error or '-'}")
            return " ".join(parts)
