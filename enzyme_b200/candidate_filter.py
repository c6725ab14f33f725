"""Tile-candidate filtering before benchmarking.

Each variant module carries a literal `__axon_tile_constraints__` manifest (the
contract of Axon's src/axon/candidate_filter.py:13-103): one record per
TILES_IN_BLOCK_* argument giving the extent it tiles, the size of one tile and
whether the block must divide the extent. The CUDA variants add an optional
`allowed` list for knobs whose legal values are not a divisibility rule (for
example GEMM pipeline depths). `select_diverse` then picks a deterministic
quality/diversity subset under a budget: the anchors (the extremes of every
axis) first, then greedily the candidate with the best mix of quality (mean
normalised log2 tile size) and distance from the picks so far, hash-seeded for
ties.
"""

from __future__ import annotations

import ast
import hashlib
import math
from collections.abc import Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

MANIFEST_NAME = "__axon_tile_constraints__"
MANIFEST_VERSION = 1


@dataclass(frozen=True, slots=True)
class TileConstraint:
    tile_arg: str
    extent: int
    tile_size: int
    require_divisible: bool
    allowed: tuple[int, ...] | None = field(default=None)

    def rejection_reason(self, value: int) -> str | None:
        if value <= 0:
            return f"{self.tile_arg}={value} is not positive"
        if self.allowed is not None and value not in self.allowed:
            return f"{self.tile_arg}={value} not in {list(self.allowed)}"
        block = self.tile_size * value
        if block > self.extent:
            return f"{self.tile_arg}={value} gives block {block} > extent {self.extent}"
        if self.require_divisible and self.extent % block:
            return f"{self.tile_arg}={value} gives block {block}, which does not divide extent {self.extent}"
        return None

    def as_record(self) -> dict[str, Any]:
        rec: dict[str, Any] = {
            "tile_arg": self.tile_arg,
            "extent": self.extent,
            "tile_size": self.tile_size,
            "require_divisible": self.require_divisible,
        }
        if self.allowed is not None:
            rec["allowed"] = list(self.allowed)
        return rec


def manifest_literal(constraints: Sequence[TileConstraint]) -> str:
    recs = tuple(c.as_record() for c in sorted(constraints, key=lambda c: c.tile_arg))
    return repr({"version": MANIFEST_VERSION, "constraints": recs})


def read_manifest(module_path: str | Path) -> tuple[TileConstraint, ...]:
    """Parse only the literal manifest assignment; anything malformed reads as
    'no constraints' (the module is then benchmarked unfiltered)."""
    path = Path(module_path)
    if not path.is_file():
        return ()
    try:
        tree = ast.parse(path.read_text(), filename=str(path))
        value = None
        for node in tree.body:
            if isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id == MANIFEST_NAME for t in node.targets
            ):
                value = ast.literal_eval(node.value)
                break
        if value is None:
            return ()
        if isinstance(value, dict):
            if value.get("version") != MANIFEST_VERSION:
                return ()
            records = value.get("constraints")
        else:
            records = value
        out = []
        for r in records:
            r = dict(r)
            if r.get("allowed") is not None:
                r["allowed"] = tuple(int(v) for v in r["allowed"])
            out.append(TileConstraint(**r))
        constraints = tuple(out)
    except (OSError, SyntaxError, ValueError, TypeError):
        return ()
    if len({c.tile_arg for c in constraints}) != len(constraints):
        return ()
    return constraints


def rejection_reason(tile_args: Sequence[str], tile_values: Sequence[int],
                     constraints: Sequence[TileConstraint]) -> str | None:
    values = dict(zip(tile_args, tile_values, strict=True))
    for c in constraints:
        v = values.get(c.tile_arg)
        if v is None:
            continue
        reason = c.rejection_reason(int(v))
        if reason is not None:
            return reason
    return None


def select_diverse(tile_values: Sequence[tuple[int, ...]], *, budget: int, seed: int) -> list[tuple[int, ...]]:
    cands = sorted(set(tile_values))
    if budget <= 0 or len(cands) <= budget:
        return cands
    width = len(cands[0])
    hi = tuple(max(c[i] for c in cands) for i in range(width))
    lo = tuple(min(c[i] for c in cands) for i in range(width))
    vec = {c: tuple(math.log2(v) / math.log2(m) if m > 1 else 0.0 for v, m in zip(c, hi)) for c in cands}

    def quality(c):
        p = vec[c]
        return sum(p) / len(p) if p else 0.0

    def tie(c):
        h = hashlib.sha256(f"{seed}:{','.join(map(str, c))}".encode()).digest()
        return int.from_bytes(h[:8], "big")

    anchors = {min(cands), max(cands)}
    for i in range(width):
        a = list(lo)
        a[i] = hi[i]
        b = list(hi)
        b[i] = lo[i]
        for t in (tuple(a), tuple(b)):
            if t in vec:
                anchors.add(t)
    chosen = sorted(anchors, key=lambda c: (-quality(c), tie(c)))[:budget]

    def dist(x, y):
        return math.sqrt(sum((a - b) ** 2 for a, b in zip(vec[x], vec[y])))

    rest = [c for c in cands if c not in chosen]
    while rest and len(chosen) < budget:
        pick = max(rest, key=lambda c: (0.65 * quality(c) + 0.35 * min(dist(c, p) for p in chosen), -tie(c)))
        chosen.append(pick)
        rest.remove(pick)
    return sorted(chosen)
