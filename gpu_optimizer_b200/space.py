"""Candidate configurations: parameter spaces and candidate identity.

The search stack of the reference (searchers, action catalog, validity
masks, surrogate) speaks in config dicts over per-task parameter spaces
(compiler/transformations/space.py:23-206).  This module keeps that
interface — same Config dict, same ParamSpec semantics (ordered discrete
choices, or a continuous [low, high] range), same ``candidate_id`` (sha1
of the sorted JSON of task, shape and config, space.py:185-191) — so
results recorded by this backend key into the reference's results database
and searchers unchanged.  The agreement is tested against the reference's
own module where it is installed.
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
    """One tunable parameter: an ordered tuple of discrete ``choices``
    (adjacent entries are neighbours), or a continuous ``low``..``high``
    range (space.py:26-58)."""

    name: str
    choices: tuple[ConfigValue, ...] | None = None
    low: float | None = None
    high: float | None = None

    def __post_init__(self) -> None:
        if (self.choices is None) == (self.low is None or self.high is None):
            raise ValueError(f"{self.name}: specify either choices or (low, high)")

    @property
    def is_continuous(self) -> bool:
        return self.choices is None

    def sample(self, rng: random.Random) -> ConfigValue:
        if self.is_continuous:
            return rng.uniform(self.low, self.high)
        return rng.choice(self.choices)

    def index_of(self, value: ConfigValue) -> int:
        if self.is_continuous:
            raise TypeError(f"{self.name} is continuous")
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

    @property
    def discrete_specs(self) -> list[ParamSpec]:
        return [s for s in self if not s.is_continuous]

    def size(self) -> int:
        """Number of discrete configurations (continuous parameters excluded)."""
        n = 1
        for s in self.discrete_specs:
            n *= len(s.choices)
        return n

    def sample(self, rng: random.Random) -> Config:
        return {s.name: s.sample(rng) for s in self}

    def grid(self, limit: int | None = None) -> list[Config]:
        """Cartesian product of the discrete parameters; continuous ones at
        their midpoint."""
        disc = self.discrete_specs
        names = [s.name for s in disc]
        out: list[Config] = []
        for combo in itertools.product(*(s.choices for s in disc)):
            cfg: Config = dict(zip(names, combo))
            for s in self:
                if s.is_continuous:
                    cfg[s.name] = (s.low + s.high) / 2.0
            out.append(cfg)
            if limit is not None and len(out) >= limit:
                break
        return out

    def validate(self, config: Config) -> None:
        for s in self:
            if s.name not in config:
                raise ValueError(f"missing param {s.name}")
            v = config[s.name]
            if s.is_continuous:
                if not (s.low <= float(v) <= s.high):
                    raise ValueError(f"{s.name}={v} outside [{s.low}, {s.high}]")
            elif v not in s.choices:
                raise ValueError(f"{s.name}={v!r} not in {s.choices}")

    def neighbors(self, config: Config) -> list[Config]:
        """Configs one discrete step away (the local-mutation neighbourhood)."""
        out = []
        for s in self.discrete_specs:
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

    def mutated(self, config: Config, provenance: str) -> Candidate:
        return Candidate(task=self.task, shape=self.shape, config=config,
                         parent_id=self.candidate_id, provenance=provenance)

    def describe(self) -> str:
        cfg = ", ".join(f"{k}={v}" for k, v in sorted(self.config.items()))
        return f"{self.task}{list(self.shape)} [{cfg}]"
