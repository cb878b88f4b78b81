"""The measured pipe / tile table (``orchestrator/assembly/pipe_table.py``): lookup
rules, forced variants, and that the planner follows the committed measurements."""

from __future__ import annotations

import json

import pytest

from metellus_b200 import configs
from metellus_b200.api.run import compile_program
from metellus_b200.orchestrator.assembly import pipe_table
from metellus_b200.orchestrator.assembly.measure_pipe_table import _variant_of


@pytest.fixture
def table(tmp_path, monkeypatch):
    doc = {"entries": [
        {"shape": [1024, 1024, 1024, 1], "us": {"ffma": 90.0, "one": 40.0, "splitk": 28.0, "pair": 35.0},
         "best": "splitk"},
        {"shape": [128, 128, 128, 1], "us": {"ffma": 6.0, "one": 9.0}, "best": "ffma"},
        {"shape": [4096, 4096, 4096, 2], "us": {"one": 900.0, "pair": 700.0}, "best": "pair"},
    ]}
    p = tmp_path / "pipe_table.json"
    p.write_text(json.dumps(doc))
    monkeypatch.setattr(pipe_table, "TABLE_PATH", p)
    pipe_table._load.cache_clear()
    yield p
    pipe_table._load.cache_clear()


def test_exact_near_and_missing(table):
    assert pipe_table.lookup(1024, 1024, 1024) == pipe_table.Pick("splitk", "table")
    assert pipe_table.lookup(1536, 1024, 800) == pipe_table.Pick("splitk", "table-near")
    assert pipe_table.lookup(4096, 4096, 4096, 1) is None          # no one-anchor entry nearby
    assert pipe_table.lookup(4096, 4096, 4096, 2).variant == "pair"
    assert pipe_table.lookup(100, 128, 200).variant == "ffma"


def test_forced_overrides_table(table):
    with pipe_table.forced("one"):
        assert pipe_table.lookup(1024, 1024, 1024) == pipe_table.Pick("one", "forced")
    with pytest.raises(ValueError):
        with pipe_table.forced("wmma"):
            pass


def test_planner_follows_table(table):
    c = configs.CONFIGS["c1"]
    (g,) = compile_program(c.build(M=1024, K=1024, N=1024, materialize=False))
    assert _variant_of(g) == "splitk"
    # the small shape is measured faster on the FFMA tile
    (g,) = compile_program(c.build(M=128, K=128, N=128, materialize=False))
    assert _variant_of(g) == "ffma"
    with pipe_table.forced("pair"):
        (g,) = compile_program(c.build(M=1024, K=1024, N=1024, materialize=False))
    assert _variant_of(g) == "pair" and g.cluster_x == 2


def test_committed_table_picks_are_used():
    """Every committed entry's fastest variant is what the planner picks for it."""
    pipe_table._load.cache_clear()
    ents = pipe_table.entries()
    if not ents:
        pytest.skip("no committed table")
    for e in ents:
        M, N, K, nb = e["shape"]
        assert e["best"] == min(e["us"], key=e["us"].get)
        assert pipe_table.lookup(M, N, K, nb).variant == e["best"]
    key = {tuple(e["shape"]): e["best"] for e in ents}
    for cfg, shape, nb in (("c1", dict(M=1024, K=1024, N=1024), 1),):
        want = key.get((shape["M"], shape["N"], shape["K"], nb))
        if want is None:
            continue
        (g,) = compile_program(configs.CONFIGS[cfg].build(**shape, materialize=False))
        assert _variant_of(g) == want
