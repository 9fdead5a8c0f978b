"""The device RNG header (splitmix64 seeds, multiply-high bounded draw and
the GF(2) jump-ahead tables) compiled for the host and checked against the
oracle's serial restatement of the reference generator."""

from __future__ import annotations

import functools
import random
import subprocess
from pathlib import Path

import pytest

from oracle import oracle

REPO = Path(__file__).resolve().parents[1]
U64 = (1 << 64) - 1


@functools.lru_cache(maxsize=None)
def checker(tmp_dir: str) -> Path:
    exe = Path(tmp_dir) / "rng_check"
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{REPO / 'fusesampleagg_b200' / 'csrc'}",
                    str(REPO / "tests" / "native" / "rng_check.cpp"), "-o", str(exe)],
                   check=True)
    return exe


@pytest.fixture(scope="module")
def run(tmp_path_factory):
    exe = checker(str(tmp_path_factory.mktemp("rng")))

    def query(lines):
        out = subprocess.run([str(exe)], input="\n".join(lines) + "\n", capture_output=True,
                             text=True, check=True).stdout.split("\n")
        return [line for line in out if line]

    return query


def test_jump_ahead_equals_serial_steps(run):
    rng = random.Random(1)
    cases = [(rng.getrandbits(64) | 1, n) for n in
             [0, 1, 2, 3, 7, 15, 16, 17, 63, 64, 100, 1023, 4096, 12345, 65535, 100_003]]
    cases += [(0x9E3779B97F4A7C15, 1 << k) for k in range(0, 18)]
    got = run([f"jump {s} {n}" for s, n in cases])
    want = [str(oracle.xorshift_advance(s, n)) for s, n in cases]
    assert got == want


def test_bounded_draw_equals_128bit_product(run):
    rng = random.Random(2)
    cases = [(rng.getrandbits(64), rng.randrange(1, 1 << 32)) for _ in range(200)]
    cases += [(U64, 1), (U64, (1 << 32) - 1), (0, 5), (1 << 63, 2)]
    got = run([f"draw {r} {b}" for r, b in cases])
    want = [str((r * b) >> 64) for r, b in cases]
    assert got == want


def test_bounded_draw_matches_oracle_generator(run):
    rng = random.Random(3)
    # oracle.bounded(state, bound) steps the state once, multiplies by the
    # xorshift* constant and draws; the header does the same in two parts.
    for _ in range(50):
        s = rng.getrandbits(64) | 1
        b = rng.randrange(1, 1 << 31)
        stepped = oracle.xorshift_advance(s, 1)
        r = (stepped * 2685821657736338717) & U64
        assert run([f"draw {r} {b}"]) == [str(oracle.bounded(s, b))]


def test_row_seeds_match_oracle(run):
    rng = random.Random(4)
    for base in [0, 1, 1234, U64, rng.getrandbits(64)]:
        root = rng.randrange(0, 1 << 31)
        got = run([f"seed {base} {root}"])[0].split()
        assert int(got[0]) == oracle.row_state(base, root, 1, 3)
        assert int(got[1]) == oracle.row_state(base, root, 0, root)


def test_chunk_start_equals_serial_steps(run):
    rng = random.Random(5)
    chunk = 64
    js = [0, 1, 2, 5, 31, 32, 33, 63, 64, 65, 100, 127, 128, 500, 1023, 1024, 1025, 4097,
          33_000, 16_000_000 // chunk]
    cases = [(rng.getrandbits(64) | 1, j) for j in js]
    got = run([f"chunk {s} {j}" for s, j in cases])
    want = [str(oracle.xorshift_advance(s, j * chunk)) for s, j in cases]
    assert got == want
    # the 2-hop draw kernel's form (one-chunk tables with the lane innermost)
    assert run([f"chunkt {s} {j}" for s, j in cases]) == want
