"""Candidate configurations: parameter spaces and candidate identity.

The search stack of the reference (searchers, action catalog, validity
masks, surrogate) speaks in config dicts over per-task parameter spaces
(compiler/transformations/space.py:23-206).  This module keeps that
interface — same Config dict, same ordered-choice ParamSpec semantics, same
``candidate_id`` (sha1 of the sorted JSON of task, shape and config,
space.py:185-191) — so results recorded by this backend key into the
reference's results database and searchers unchanged.
"""

from __future__ import annotations

import hashlib
import itertools
import json
import random
from collections.abc import Iterator, Sequence
from dataclasses import dataclass, field

ConfigValue = int | float | str
Config = dict[str, ConfigValue]


@dataclass(frozen=True)
class ParamSpec:
    """One tunable parameter with an ordered tuple of discrete choices."""

    name: str
    choices: tuple[ConfigValue, ...]

    def sample(self, rng: random.Random) -> ConfigValue:
        return rng.choice(self.choices)

    def index_of(self, value: ConfigValue) -> int:
        return self.choices.index(value)


class ParamSpace:
    """Ordered collection of ParamSpecs (space.py:61-130)."""

    def __init__(self, specs: Sequence[ParamSpec], name: str = "space") -> None:
        self.name = name
        self.specs: dict[str, ParamSpec] = {s.name: s for s in specs}
        if len(self.specs) != len(specs):
            raise ValueError("duplicate parameter names")

    def __iter__(self) -> Iterator[ParamSpec]:
        return iter(self.specs.values())

    def __getitem__(self, name: str) -> ParamSpec:
        return self.specs[name]

    def __contains__(self, name: str) -> bool:
        return name in self.specs

    def size(self) -> int:
        n = 1
        for s in self:
            n *= len(s.choices)
        return n

    def sample(self, rng: random.Random) -> Config:
        return {s.name: s.sample(rng) for s in self}

    def grid(self, limit: int | None = None) -> list[Config]:
        names = [s.name for s in self]
        out: list[Config] = []
        for combo in itertools.product(*(s.choices for s in self)):
            out.append(dict(zip(names, combo)))
            if limit is not None and len(out) >= limit:
                break
        return out

    def validate(self, config: Config) -> None:
        for s in self:
            if s.name not in config:
                raise ValueError(f"missing param {s.name}")
            if config[s.name] not in s.choices:
                raise ValueError(f"{s.name}={config[s.name]!r} not in {s.choices}")

    def neighbors(self, config: Config) -> list[Config]:
        out = []
        for s in self:
            idx = s.index_of(config[s.name])
            for d in (-1, 1):
                j = idx + d
                if 0 <= j < len(s.choices):
                    cfg = dict(config)
                    cfg[s.name] = s.choices[j]
                    out.append(cfg)
        return out


@dataclass
class Candidate:
    """A concrete configuration for one task instance (space.py:171-206)."""

    task: str
    shape: tuple[int, ...]
    config: Config = field(default_factory=dict)
    parent_id: str | None = None
    provenance: str = "manual"
    predicted_ms: float | None = None
    predicted_std: float | None = None

    @property
    def candidate_id(self) -> str:
        payload = json.dumps({"task": self.task, "shape": list(self.shape),
                              "config": self.config}, sort_keys=True, default=str)
        return hashlib.sha1(payload.encode()).hexdigest()[:16]

    @property
    def dtype(self) -> str:
        return str(self.config.get("dtype", "float32"))

    def describe(self) -> str:
        cfg = ", ".join(f"{k}={v}" for k, v in sorted(self.config.items()))
        return f"{self.task}{list(self.shape)} [{cfg}]"
