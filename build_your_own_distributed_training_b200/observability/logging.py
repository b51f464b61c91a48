"""One JSON object per line: ``ts, level, rank, run_id, event, **fields``.

``info``/``metric`` print on rank 0 only; ``warning``/``error`` on every rank
(schema and gating of ``src/observability/logging.py:28-98``).
"""

from __future__ import annotations

import json
import sys
import time
from dataclasses import asdict, is_dataclass
from typing import Any


class RankLogger:
    def __init__(self, rank: int, run_id: str, stream: Any = None) -> None:
        self.rank, self.run_id = rank, run_id
        self.stream = stream if stream is not None else sys.stdout
        self._t0 = time.time()

    def _emit(self, level: str, event: str, rank0_only: bool, **fields: Any) -> None:
        if rank0_only and self.rank != 0:
            return
        rec: dict[str, Any] = {"ts": round(time.time() - self._t0, 4), "level": level,
                               "rank": self.rank, "run_id": self.run_id, "event": event}
        rec.update({k: _jsonable(v) for k, v in fields.items()})
        self.stream.write(json.dumps(rec) + "\n")
        self.stream.flush()

    def info(self, event: str, **fields: Any) -> None:
        self._emit("INFO", event, True, **fields)

    def metric(self, event: str, **fields: Any) -> None:
        self._emit("METRIC", event, True, **fields)

    def warning(self, event: str, **fields: Any) -> None:
        self._emit("WARNING", event, False, **fields)

    def error(self, event: str, **fields: Any) -> None:
        self._emit("ERROR", event, False, **fields)


def _jsonable(v: Any) -> Any:
    if is_dataclass(v) and not isinstance(v, type):
        return {k: _jsonable(x) for k, x in asdict(v).items()}
    if v is None or isinstance(v, (str, int, float, bool)):
        return v
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    return str(v)


def build_logger(rank: int, run_id: str, stream: Any | None = None) -> RankLogger:
    return RankLogger(rank, run_id, stream)
