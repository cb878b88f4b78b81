"""Generate the golden fixtures from the reference source (run where the reference is
checked out; the fixtures are committed, so tests never need the reference):

    python tests/golden/make_golden.py /path/to/metellus

1. ``plans.json``: for every program in ``programs.PROGRAMS``, the reference's own
   ``fuse -> assemble -> alias_group`` plan (src/api/run.py:37-41) at its 32 KB cap:
   per kernel the strategy, absorbed op outputs, bindings, dims and post-alias
   threadgroup bytes. The reference imports its Metal backend at module load
   (runtime/program.py:7); a no-op stand-in module is put on the path for planning,
   and nothing is executed.
2. ``elementwise_ops.json``: the reference's elementwise expression table
   (compute/elementwise/elementwise.py:18-55) evaluated in IEEE fp32 on a fixed set of
   edge-case inputs (+-0, +-inf, NaN, subnormals, large and small magnitudes),
   including the comparison -> 1.0/0.0 wrapping (assembly/expressions.py:43-48). The
   MSL expression strings are read from the reference and interpreted by a small C
   expression evaluator below; results are stored as fp32 bit patterns.
"""

from __future__ import annotations

import importlib
import json
import os
import re
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import programs  # noqa: E402

STUB = '''
def create_buffer(n): return 1
def release_buffer(h): return True
def buffer_size(h): return 0
def write_buffer(h, a): pass
def read_buffer(h, a): pass
def fill_buffer(h, v): pass
def run_kernel(*a, **k): return {"time_ms": 0.0}
'''


def load_reference(ref_root: Path):
    tmp = Path(tempfile.mkdtemp())
    (tmp / "metal_backend.py").write_text(STUB)
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(tmp), str(ref_root / "src")]
    mods = {}
    for m in ("orchestrator", "orchestrator.fusion", "orchestrator.assembly", "orchestrator.aliasing",
              "compute.elementwise.elementwise"):
        mods[m] = importlib.import_module(m)
    return mods


def make_plans(mods) -> dict:
    Operations = mods["orchestrator"].Operations
    fuse = mods["orchestrator.fusion"].fuse
    assemble = mods["orchestrator.assembly"].assemble
    aliasing = mods["orchestrator.aliasing"]
    out = {}
    for name, spec in programs.PROGRAMS.items():
        ops = Operations()
        spec(ops)
        groups = []
        for v in fuse(ops.build()):
            g = aliasing.alias_group(assemble(v))
            groups.append({
                "strategy": str(g.strategy.value),
                "ops": [op.out.name for op in g.ops],
                "bindings": list(g.bindings),
                "dims": list(g.dims),
                "tgmem_bytes": int(aliasing.compute_group_budget(g).size_bytes),
            })
        out[name] = {"cap_bytes": int(aliasing.TGMEM_CAP_BYTES), "groups": groups}
    return out


# -- a tiny C expression evaluator over numpy float32 -----------------------------------

_TOK = re.compile(r"\s*(?:(\d+\.\d*f?|\d+f?)|([A-Za-z_]\w*)|(>=|<=|==|!=|[-+*/()?:,<>]))")


def _tokens(s: str):
    pos, out = 0, []
    while pos < len(s):
        m = _TOK.match(s, pos)
        if not m or m.end() == pos:
            if s[pos:].strip() == "":
                break
            raise ValueError(f"cannot tokenize {s[pos:]!r}")
        pos = m.end()
        num, ident, op = m.groups()
        out.append(("num", num) if num else ("id", ident) if ident else ("op", op))
    return out


class _Eval:
    F32 = np.float32
    FUNCS = {
        "fabs": np.abs, "exp": np.exp, "log": np.log, "sqrt": np.sqrt, "sin": np.sin, "cos": np.cos,
        "floor": np.floor, "ceil": np.ceil, "copysign": np.copysign, "fmax": np.fmax, "fmin": np.fmin,
        "pow": np.power,
    }

    def __init__(self, expr: str, env: dict):
        self.t = _tokens(expr)
        self.i = 0
        self.env = env

    def peek(self):
        return self.t[self.i] if self.i < len(self.t) else (None, None)

    def take(self, v=None):
        tok = self.peek()
        if v is not None and tok[1] != v:
            raise ValueError(f"expected {v!r}, got {tok!r}")
        self.i += 1
        return tok

    def parse(self):
        with np.errstate(all="ignore"):
            r = self.ternary()
        if self.i != len(self.t):
            raise ValueError("trailing tokens")
        return r

    def ternary(self):
        c = self.equality()
        if self.peek()[1] == "?":
            self.take("?")
            a = self.ternary()
            self.take(":")
            b = self.ternary()
            return np.where(np.asarray(c, bool) if np.asarray(c).dtype == bool else (np.asarray(c) != 0), a, b).astype(self.F32)
        return c

    def equality(self):
        a = self.relational()
        while self.peek()[1] in ("==", "!="):
            op = self.take()[1]
            b = self.relational()
            a = (a == b) if op == "==" else (a != b)
        return a

    def relational(self):
        a = self.additive()
        while self.peek()[1] in ("<", ">", "<=", ">="):
            op = self.take()[1]
            b = self.additive()
            a = {"<": np.less, ">": np.greater, "<=": np.less_equal, ">=": np.greater_equal}[op](a, b)
        return a

    def additive(self):
        a = self.mult()
        while self.peek()[1] in ("+", "-"):
            op = self.take()[1]
            b = self.mult()
            a = (a + b if op == "+" else a - b).astype(self.F32)
        return a

    def mult(self):
        a = self.unary()
        while self.peek()[1] in ("*", "/"):
            op = self.take()[1]
            b = self.unary()
            a = (a * b if op == "*" else a / b).astype(self.F32)
        return a

    def unary(self):
        if self.peek()[1] == "-":
            self.take("-")
            return (-self.unary()).astype(self.F32)
        return self.primary()

    def primary(self):
        kind, v = self.take()
        if kind == "num":
            return self.F32(float(v.rstrip("f")))
        if kind == "id":
            if self.peek()[1] == "(":
                self.take("(")
                args = [self.ternary()]
                while self.peek()[1] == ",":
                    self.take(",")
                    args.append(self.ternary())
                self.take(")")
                return np.asarray(self.FUNCS[v](*[np.asarray(a, self.F32) for a in args]), self.F32)
            return self.env[v]
        if v == "(":
            r = self.ternary()
            self.take(")")
            return r
        raise ValueError(f"unexpected token {v!r}")


def edge_inputs() -> np.ndarray:
    vals = [0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 2.0, -3.0, 1e-3, -1e-3, 1e-30, 1e-40, -1e-40, 3.0e38,
            -3.0e38, 88.0, -88.0, 100.0, -100.0, 1e4, 0.3, -0.7, 7.25, np.inf, -np.inf, np.nan, 1e-8, 20.0]
    return np.array(vals, dtype=np.float32)


def make_elementwise(mods) -> dict:
    ew = mods["compute.elementwise.elementwise"]
    xs = edge_inputs()
    n = len(xs)
    X = np.repeat(xs, n)
    Y = np.tile(xs, n)
    C = np.tile(np.array([0.0, 1.0, -0.0, np.nan], np.float32), (n * n) // 4 + 1)[: n * n]
    out = {"inputs_hex": [f"{int(v):08x}" for v in xs.view(np.uint32)], "ops": {}}
    for table, arity in ((ew.UNARY_EXPRESSIONS, 1), (ew.BINARY_EXPRESSIONS, 2), (ew.TERNARY_EXPRESSIONS, 3)):
        for op, expr in table.items():
            env = {"x": xs if arity == 1 else X, "y": Y, "cond": C}
            r = _Eval(expr, env).parse()
            r = np.asarray(r)
            if r.dtype == bool or op in ew.COMPARISON_OPS:
                r = np.where(np.asarray(r, bool), np.float32(1), np.float32(0))
            r = np.broadcast_to(np.asarray(r, np.float32), env["x"].shape)
            out["ops"][op] = {"arity": arity, "expr": expr,
                              "out_hex": [f"{int(v):08x}" for v in np.ascontiguousarray(r).view(np.uint32)]}
    out["cond_hex"] = [f"{int(v):08x}" for v in C.view(np.uint32)]
    return out


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("METELLUS_REFERENCE", ""))
    if not (ref / "src" / "orchestrator").exists():
        raise SystemExit("usage: make_golden.py <reference checkout>")
    mods = load_reference(ref)
    (HERE / "plans.json").write_text(json.dumps(make_plans(mods), indent=1))
    (HERE / "elementwise_ops.json").write_text(json.dumps(make_elementwise(mods)))
    print("wrote", HERE / "plans.json", HERE / "elementwise_ops.json")


if __name__ == "__main__":
    main()
