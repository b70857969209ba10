"""Modifier lifecycle, session and state (host-side control flow around the kernels).

Mirrors ``ModifierBase`` (src/LLMCompressorSharp.Core/Modifiers/ModifierBase.cs:18-181),
``TargetMatcher`` (TargetMatcher.cs:22-86), ``CompressionState``
(Compression/CompressionState.cs:17-65) and ``CompressionSession``
(Compression/CompressionSession.cs:18-118).  No arithmetic happens here.
"""

from __future__ import annotations

import enum
import re
from typing import Iterable

import torch

from .errors import ArgumentError, LlmcError


class ModifierLifecycleError(LlmcError):
    """ModifierLifecycleException."""


class SessionStatus(enum.Enum):
    NOT_STARTED = 0
    RUNNING = 1
    COMPLETED = 2
    FAILED = 3


class CompressionState:
    """CompressionState.cs:17-65."""

    def __init__(self, named_weights: dict[str, torch.Tensor], rng_seed: int = 0):
        if named_weights is None:
            raise ArgumentError("namedWeights must not be null")
        self.named_weights: dict[str, torch.Tensor] = dict(named_weights)
        self.current_batch = None
        self.current_batch_index = 0
        self.layer_activations: dict[str, torch.Tensor] | None = None
        self.named_modules: dict[str, torch.nn.Module] | None = None
        self.rng_seed = rng_seed
        # Packed outputs of quantising modifiers: name -> dict(codes, scales, zero_points, ...)
        self.compressed: dict[str, dict] = {}


class TargetMatcher:
    """TargetMatcher.cs:22-86: '*' globs, ignore wins, empty targets match everything."""

    @staticmethod
    def _matches_pattern(name: str, pattern: str) -> bool:
        if not pattern:
            return False
        if "*" not in pattern:
            return name == pattern
        rx = "^" + re.escape(pattern).replace("\\*", ".*") + "$"
        return re.match(rx, name) is not None

    @staticmethod
    def matches(name: str, targets, ignore) -> bool:
        for p in ignore:
            if TargetMatcher._matches_pattern(name, p):
                return False
        if not targets:
            return True
        return any(TargetMatcher._matches_pattern(name, p) for p in targets)

    @staticmethod
    def filter(names: Iterable[str], targets, ignore):
        return [n for n in names if TargetMatcher.matches(n, targets, ignore)]


class ModifierBase:
    """ModifierBase.cs:18-181 — Initialize -> OnStart -> OnBatch* -> OnEnd -> Finalize."""

    def __init__(self, name: str, targets=None, ignore=None):
        if not name or not name.strip():
            raise ArgumentError("name must not be empty")
        self.name = name
        self.targets = list(targets or [])
        self.ignore = list(ignore or [])
        self._initialized = self._started = self._ended = self._finalized = False

    def initialize(self, state: CompressionState):
        if self._initialized:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was initialized twice.")
        self._initialized = True
        self.on_initialize(state)

    def on_start(self, state: CompressionState):
        self._ensure_initialized()
        if self._started:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was started twice.")
        self._started = True
        self.on_start_core(state)

    def on_batch(self, state: CompressionState):
        self._ensure_started()
        if self._ended:
            raise ModifierLifecycleError(f"Modifier '{self.name}' received a batch after OnEnd.")
        self.on_batch_core(state)

    def on_end(self, state: CompressionState):
        self._ensure_started()
        if self._ended:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was ended twice.")
        self._ended = True
        self.on_end_core(state)

    def finalize(self, state: CompressionState):
        if not self._initialized:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was finalized before being initialized.")
        if self._finalized:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was finalized twice.")
        self._finalized = True
        self.on_finalize_core(state)

    # hooks
    def on_initialize(self, state):
        pass

    def on_start_core(self, state):
        pass

    def on_batch_core(self, state):
        pass

    def on_end_core(self, state):
        raise NotImplementedError

    def on_finalize_core(self, state):
        pass

    def targeted_names(self, state: CompressionState):
        return TargetMatcher.filter(list(state.named_weights.keys()), self.targets, self.ignore)

    def _ensure_initialized(self):
        if not self._initialized:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was used before Initialize.")

    def _ensure_started(self):
        self._ensure_initialized()
        if not self._started:
            raise ModifierLifecycleError(f"Modifier '{self.name}' was used before OnStart.")


class CompressionSession:
    """CompressionSession.cs:18-118: runs the lifecycle; on failure records it and still
    finalises every initialised modifier."""

    def __init__(self, modifiers):
        if modifiers is None:
            raise ArgumentError("modifiers must not be null")
        self.modifiers = list(modifiers)
        self._initialized = []
        self.status = SessionStatus.NOT_STARTED
        self.failure: BaseException | None = None

    def run(self, state: CompressionState, batches) -> SessionStatus:
        if state is None or batches is None:
            raise ArgumentError("state and batches must not be null")
        if self.status != SessionStatus.NOT_STARTED:
            raise ModifierLifecycleError("CompressionSession.Run may only be called once.")
        self.status = SessionStatus.RUNNING
        try:
            for m in self.modifiers:
                m.initialize(state)
                self._initialized.append(m)
            for m in self.modifiers:
                m.on_start(state)
            for i, b in enumerate(batches):
                state.current_batch = b
                state.current_batch_index = i
                for m in self.modifiers:
                    m.on_batch(state)
            state.current_batch = None
            for m in self.modifiers:
                m.on_end(state)
            self.status = SessionStatus.COMPLETED
        except Exception as ex:  # noqa: BLE001 — the reference catches every exception
            self.status = SessionStatus.FAILED
            self.failure = ex
        finally:
            for m in self._initialized:
                try:
                    m.finalize(state)
                except Exception:
                    if self.status != SessionStatus.FAILED:
                        raise
        return self.status
