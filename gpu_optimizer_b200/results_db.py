"""B200 measurement fields in the reference's results database.

The reference persists every ``BenchmarkResult`` in SQLite through
``BenchmarkDB.insert_result`` (benchmarks/db.py:20-89 schema, :113-138
insert), and the dashboard shows a candidate's kernel source through
``render_source`` (server/api/main.py:170-188).  This backend's results
carry fields the reference's ``results`` table has no columns for: the
achieved GB/s or TFLOP/s of the task's algorithmic work, its fraction of
the measured peak, the kernel instantiation, the device and worker that
measured it, and the two relative-error figures.

``B200ResultsDB`` leaves the reference's schema unchanged and keeps those
fields in an added table, ``b200_results``, keyed by the reference's
result row id.  It wraps any object with the reference's
``BenchmarkDB`` interface (``path`` and ``insert_result``), so results
stay readable by the unchanged dashboard and surrogate-training code.
Writes are made only by the process that opened it -- the search's
coordinator; device workers send their results to the coordinator, as
SQLite is written by one process (benchmarks/db.py:101-110).
"""

from __future__ import annotations

import os
import sqlite3
from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from pathlib import Path

B200_SCHEMA = """
CREATE TABLE IF NOT EXISTS b200_results (
    result_id INTEGER PRIMARY KEY,
    candidate_id TEXT NOT NULL,
    achieved REAL,
    achieved_unit TEXT,
    roofline_fraction REAL,
    kernel TEXT,
    device_index INTEGER,
    worker_id INTEGER,
    rel_err_floored REAL,
    rel_err_normwise REAL
);
CREATE INDEX IF NOT EXISTS idx_b200_candidate ON b200_results(candidate_id);
"""

B200_FIELDS = ("achieved", "achieved_unit", "roofline_fraction", "kernel", "device_index",
               "worker_id", "rel_err_floored", "rel_err_normwise")


class B200ResultsDB:
    """The reference's results database plus the ``b200_results`` table."""

    def __init__(self, base) -> None:
        self.base = base
        self.path = Path(base.path)
        self._owner = os.getpid()
        with self._conn() as con:
            con.executescript(B200_SCHEMA)

    @contextmanager
    def _conn(self) -> Iterator[sqlite3.Connection]:
        con = sqlite3.connect(self.path, timeout=30.0)
        con.row_factory = sqlite3.Row
        try:
            yield con
            con.commit()
        finally:
            con.close()

    def __getattr__(self, name: str):
        # runs, iterations and queries: the reference database's own methods
        base = self.__dict__.get("base")
        if base is None:
            raise AttributeError(name)
        return getattr(base, name)

    def insert_result(self, r, run_id: str | None = None) -> int:
        """Insert through the reference's ``insert_result``, then the B200
        fields under the returned row id.  Coordinator only."""
        if os.getpid() != self._owner:
            raise RuntimeError("results are written by the coordinator process only")
        rid = int(self.base.insert_result(r, run_id=run_id))
        rep = getattr(r, "correctness", None)
        row = (rid, r.candidate_id, float(getattr(r, "achieved", 0.0)),
               str(getattr(r, "achieved_unit", "")),
               float(getattr(r, "roofline_fraction", 0.0)), str(getattr(r, "kernel", "")),
               int(getattr(r, "device_index", 0)), int(getattr(r, "worker_id", 0)),
               getattr(rep, "rel_err_floored", None) if rep is not None else None,
               getattr(rep, "rel_err_normwise", None) if rep is not None else None)
        with self._conn() as con:
            con.execute("INSERT INTO b200_results (result_id, candidate_id, "
                        + ", ".join(B200_FIELDS) + ") VALUES (?,?,?,?,?,?,?,?,?,?)", row)
        return rid

    def insert_many(self, results: Sequence, run_id: str | None = None) -> list[int]:
        return [self.insert_result(r, run_id) for r in results]

    def fetch(self, candidate_id: str | None = None, run_id: str | None = None,
              limit: int = 1000) -> list[dict]:
        """Result rows joined with their B200 fields (newest first)."""
        q = ("SELECT r.*, " + ", ".join(f"b.{f}" for f in B200_FIELDS)
             + " FROM results r LEFT JOIN b200_results b ON b.result_id = r.id")
        where, args = [], []
        if candidate_id is not None:
            where.append("r.candidate_id = ?")
            args.append(candidate_id)
        if run_id is not None:
            where.append("r.run_id = ?")
            args.append(run_id)
        if where:
            q += " WHERE " + " AND ".join(where)
        q += " ORDER BY r.id DESC LIMIT ?"
        args.append(limit)
        with self._conn() as con:
            return [dict(row) for row in con.execute(q, args).fetchall()]

    def candidate_source(self, candidate_id: str) -> dict:
        """The dashboard's source view (server/api/main.py:170-188) for this
        backend: the CUDA source of the kernel family with the resolved
        configuration, plus the B200 fields of the latest result."""
        import json

        from .runner import render_source

        rows = self.fetch(candidate_id=candidate_id, limit=1)
        if not rows:
            raise KeyError(f"candidate {candidate_id} not found")
        row = rows[0]
        config = json.loads(row["config"])
        shape = tuple(json.loads(row["shape"]))
        return {"candidate_id": candidate_id, "task": row["task"], "shape": list(shape),
                "config": config, "engine": row["engine"], "status": row["status"],
                "latency_ms": row["latency_median_ms"],
                **{f: row[f] for f in B200_FIELDS},
                "source": render_source(row["task"], config, shape)}
