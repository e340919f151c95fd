"""Shared helpers of the tests: the splitmix64 generator and the conformance vectors."""

from __future__ import annotations

import csv
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"
MASK64 = (1 << 64) - 1


def splitmix64(state: list[int]) -> int:
    """The splitmix64 generator (Steele, Lea, Flood 2014), as the reference tests use it
    (crates/taco-coder/tests/common/mod.rs:10). `state` is a one-element list."""
    state[0] = (state[0] + 0x9E3779B97F4A7C15) & MASK64
    z = state[0]
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def vectors() -> list[dict]:
    """The rows of conformance/v2/vectors.tsv whose files are in tests/golden."""
    rows = []
    with open(GOLDEN / "vectors.tsv") as f:
        lines = [ln for ln in f if not ln.startswith("#")]
    header = ["name", "profile", "block_size", "overlap", "input_len", "input_sha256", "container_len",
              "container_sha256", "block_kinds"]
    for r in csv.reader(lines, delimiter="\t"):
        d = dict(zip(header, r))
        if (GOLDEN / (d["name"] + ".taco")).exists():
            rows.append(d)
    return rows


def tiny_bytes() -> bytes:
    return (GOLDEN / "tiny.hsm").read_bytes()
