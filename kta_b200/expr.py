"""The shape / min_work expression language of case files.

Semantics follow src/kta/core/expr.py (an ``ast``-parsed subset of Python; ``eval`` is never
used): arithmetic ``+ - * / // % **``, unary minus, comparisons, conditional expressions and
the functions min, max, abs, ceil, floor, ceil_div, log2, is_pow2. Free names must be declared
shape variables; ``case.<name>`` reads the case's shape (used by ``params.min_work``).
Only the arithmetic subset this path needs is implemented here.
"""

from __future__ import annotations

import ast
import math
import operator
from collections.abc import Callable, Mapping
from typing import Any


class ExprError(ValueError):
    """Syntax, free-variable or evaluation error in an expression."""


def _ceil_div(a: Any, b: Any) -> int:
    if b == 0:
        raise ExprError("ceil_div by zero")
    return -(-int(a) // int(b))


def _log2(x: Any) -> float:
    if x <= 0:
        raise ExprError(f"log2 of non-positive value {x!r}")
    return math.log2(x)


def _is_pow2(x: Any) -> bool:
    return isinstance(x, int) and not isinstance(x, bool) and x > 0 and x & (x - 1) == 0


FUNCTIONS: dict[str, Callable[..., Any]] = {
    "min": min,
    "max": max,
    "abs": abs,
    "ceil": math.ceil,
    "floor": math.floor,
    "ceil_div": _ceil_div,
    "log2": _log2,
    "is_pow2": _is_pow2,
}

_BIN: dict[type[ast.operator], Callable[[Any, Any], Any]] = {
    ast.Add: operator.add,
    ast.Sub: operator.sub,
    ast.Mult: operator.mul,
    ast.Div: operator.truediv,
    ast.FloorDiv: operator.floordiv,
    ast.Mod: operator.mod,
    ast.Pow: operator.pow,
}
_CMP: dict[type[ast.cmpop], Callable[[Any, Any], bool]] = {
    ast.Lt: operator.lt,
    ast.LtE: operator.le,
    ast.Gt: operator.gt,
    ast.GtE: operator.ge,
    ast.Eq: operator.eq,
    ast.NotEq: operator.ne,
}
ROOTS = ("case",)


class Expr:
    def __init__(self, src: str, tree: ast.expr) -> None:
        self.src = src
        self._tree = tree

    @staticmethod
    def parse(src: str, declared: set[str] | None = None) -> Expr:
        declared = set(declared or ())
        try:
            tree = ast.parse(str(src).strip(), mode="eval").body
        except SyntaxError as exc:
            raise ExprError(f"syntax error in {src!r}: {exc.msg}") from exc
        for node in ast.walk(tree):
            if isinstance(node, ast.Name) and node.id not in declared and node.id not in ROOTS \
                    and node.id not in FUNCTIONS:
                raise ExprError(f"undeclared name {node.id!r} in {src!r}")
            if isinstance(node, ast.Attribute):
                if not isinstance(node.value, ast.Name) or node.value.id not in ROOTS:
                    raise ExprError(f"attribute access outside {ROOTS} in {src!r}")
            if isinstance(node, ast.Call) and (
                not isinstance(node.func, ast.Name) or node.func.id not in FUNCTIONS
            ):
                raise ExprError(f"unknown function in {src!r}")
        return Expr(src, tree)

    def eval(self, env: Mapping[str, Any] | None = None, case: Mapping[str, Any] | None = None
             ) -> Any:
        env = dict(env or {})
        case = dict(case or {})
        return self._run(self._tree, env, case)

    def _run(self, node: ast.expr, env: dict[str, Any], case: dict[str, Any]) -> Any:
        match node:
            case ast.Constant(value=v):
                return v
            case ast.Name(id=name):
                if name not in env:
                    raise ExprError(f"no value for {name!r} in {self.src!r}")
                return env[name]
            case ast.Attribute(attr=attr):
                if attr not in case:
                    raise ExprError(f"no value for case.{attr} in {self.src!r}")
                return case[attr]
            case ast.BinOp(left=left, op=op, right=right):
                fn = _BIN.get(type(op))
                if fn is None:
                    raise ExprError(f"operator {type(op).__name__} not allowed")
                a, b = self._run(left, env, case), self._run(right, env, case)
                if isinstance(op, ast.Pow) and abs(b) > 64:
                    raise ExprError("exponent too large")
                return fn(a, b)
            case ast.UnaryOp(op=ast.USub(), operand=x):
                return -self._run(x, env, case)
            case ast.UnaryOp(op=ast.UAdd(), operand=x):
                return +self._run(x, env, case)
            case ast.Compare(left=left, ops=ops, comparators=comps):
                a = self._run(left, env, case)
                for op, c in zip(ops, comps):
                    b = self._run(c, env, case)
                    if not _CMP[type(op)](a, b):
                        return False
                    a = b
                return True
            case ast.IfExp(test=t, body=b, orelse=o):
                return self._run(b if self._run(t, env, case) else o, env, case)
            case ast.Call(func=ast.Name(id=fname), args=args):
                return FUNCTIONS[fname](*(self._run(a, env, case) for a in args))
        raise ExprError(f"unsupported expression in {self.src!r}")
