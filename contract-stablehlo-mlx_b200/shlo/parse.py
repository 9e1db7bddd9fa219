"""StablehloMlx/Parse.lean restated: a dependency-free reader for StableHLO text.

It reads the generic operation form (``%r = "stablehlo.add"(%a, %b) {attrs} :
(T, T) -> T``), with regions for ``while``, ``reduce`` and other bodies
(``"stablehlo.while"(%a) ({ ^bb0(%x: T): ... "stablehlo.return"(%y) : (T) -> ()
}, { ... }) : (T) -> T``), inside ``module { func.func ... }``, plus the printed
terminators ``func.return %a, %b : T, T`` / ``return``. Multi-result ops define
``%w:2`` and are read as ``%w#0``, ``%w#1`` (Parse.lean:76-93, 178-205).

Attribute values are kept as raw text (Parse.lean:124-145); the lowering reads
them as the Lean lowering does.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from . import lower as L


class ParseError(ValueError):
    pass


@dataclass
class Block:
    """A region's one block: its arguments, ops and terminator operands."""
    args: List[Tuple[str, L.Ty]] = field(default_factory=list)
    ops: List[L.Op] = field(default_factory=list)
    ret: List[str] = field(default_factory=list)


@dataclass
class FuncDef:
    name: str
    body: Block
    out_tys: List[L.Ty]

    # the fields the executor reads (Ast.lean's Func)
    @property
    def args(self):
        return self.body.args

    @property
    def ops(self):
        return self.body.ops

    @property
    def ret(self):
        return self.body.ret


def _id_char(c: str) -> bool:
    return c.isalnum() or c in "_.$-"


class Reader:
    def __init__(self, text: str):
        self.s = text
        self.i = 0

    # ---- characters ----

    def peek(self) -> Optional[str]:
        return self.s[self.i] if self.i < len(self.s) else None

    def fail(self, msg: str):
        raise ParseError("parse error at %d: %s; next: %r" % (self.i, msg, self.s[self.i:self.i + 60]))

    def ws(self) -> None:
        while self.i < len(self.s):
            c = self.s[self.i]
            if c in " \t\r\n":
                self.i += 1
            elif self.s.startswith("//", self.i):
                j = self.s.find("\n", self.i)
                self.i = len(self.s) if j < 0 else j
            else:
                break

    def try_lit(self, lit: str) -> bool:
        self.ws()
        if self.s.startswith(lit, self.i):
            self.i += len(lit)
            return True
        return False

    def lit(self, lit: str) -> None:
        if not self.try_lit(lit):
            self.fail("expected %r" % lit)

    def take_while(self, pred) -> str:
        j = self.i
        while self.i < len(self.s) and pred(self.s[self.i]):
            self.i += 1
        return self.s[j:self.i]

    # ---- pieces ----

    def ssa(self) -> Tuple[str, Optional[int]]:
        """``%name``, ``%name#k`` (a use of one result) or ``%name:n`` (a definition of n)."""
        self.ws()
        if self.peek() != "%":
            self.fail("expected %")
        self.i += 1
        name = "%" + self.take_while(_id_char)
        if self.peek() == "#":
            self.i += 1
            return name + "#" + self.take_while(str.isdigit), None
        if self.peek() == ":" and self.i + 1 < len(self.s) and self.s[self.i + 1].isdigit():
            self.i += 1
            return name, int(self.take_while(str.isdigit))
        return name, None

    def ty(self) -> L.Ty:
        self.ws()
        if self.try_lit("tensor<"):
            dims = []
            while True:
                d = self.take_while(str.isdigit)
                if not d:
                    el = self.take_while(lambda c: c != ">")
                    break
                dims.append(int(d))
                if self.peek() != "x":
                    self.fail("expected x in a tensor type")
                self.i += 1
            self.lit(">")
            return L.Ty(tuple(dims), el)
        el = self.take_while(_id_char)
        if not el:
            self.fail("expected a type")
        return L.Ty((), el)

    def sep_by(self, item, close: str) -> list:
        if self.try_lit(close):
            return []
        xs = [item()]
        while self.try_lit(","):
            xs.append(item())
        self.lit(close)
        return xs

    def ty_list(self) -> List[L.Ty]:
        if self.try_lit("("):
            return self.sep_by(self.ty, ")")
        return [self.ty()]

    def raw_value(self) -> str:
        """One attribute value's text, up to a top-level ``,`` or ``}``."""
        self.ws()
        out, depth = [], 0
        while self.i < len(self.s):
            c = self.s[self.i]
            if depth == 0 and c in ",}":
                break
            if c == '"':
                j = self.s.find('"', self.i + 1)
                j = len(self.s) - 1 if j < 0 else j
                out.append(self.s[self.i:j + 1])
                self.i = j + 1
                continue
            if c in "([{<":
                depth += 1
            elif c in ")]}>":
                if not (c == ">" and out and out[-1].endswith("-")):  # `->` is an arrow
                    depth -= 1
            out.append(c)
            self.i += 1
        return "".join(out).strip()

    def attr_dict(self) -> dict:
        self.lit("{")

        def kv():
            self.ws()
            k = self.take_while(_id_char)
            if not k:
                self.fail("expected an attribute name")
            if self.try_lit("="):
                return k, self.raw_value()
            return k, "unit"
        return dict(self.sep_by(kv, "}"))

    # ---- blocks and ops ----

    def block(self) -> Block:
        self.lit("{")
        b = Block()
        if self.try_lit("^"):
            self.take_while(_id_char)
            if self.try_lit("("):
                def arg():
                    n = self.ssa()[0]
                    self.lit(":")
                    return n, self.ty()
                b.args = self.sep_by(arg, ")")
            self.lit(":")
        while not self.try_lit("}"):
            o = self.op()
            if o.name in ("stablehlo.return", "func.return", "return"):
                b.ret = list(o.operands)
            else:
                b.ops.append(o)
        return b

    def op(self) -> L.Op:
        self.ws()
        results = []
        if self.peek() == "%":
            defs = [self.ssa()]
            while self.try_lit(","):
                defs.append(self.ssa())
            self.lit("=")
            for n, cnt in defs:
                results += ["%s#%d" % (n, k) for k in range(cnt)] if cnt is not None else [n]
        self.ws()
        if self.peek() == '"':
            self.i += 1
            name = self.take_while(lambda c: c != '"')
            self.i += 1
            self.lit("(")
            operands = self.sep_by(lambda: self.ssa()[0], ")")
            regions = self.sep_by(self.block, ")") if self.try_lit("(") else []
            self.ws()
            attrs = self.attr_dict() if self.peek() == "{" else {}
            self.lit(":")
            self.lit("(")
            ins = self.sep_by(self.ty, ")")
            self.lit("->")
            outs = self.ty_list()
            # a multi-result op defined by one bare name: its results are name#k
            if len(results) == 1 and len(outs) > 1:
                results = ["%s#%d" % (results[0], k) for k in range(len(outs))]
            return L.Op(name, operands, results, attrs, ins, outs, regions)
        # the printed terminators: `func.return %a, %b : T, T` / `return %a : T`
        name = self.take_while(_id_char)
        if name in ("func.return", "return", "stablehlo.return"):
            operands = []
            self.ws()
            if self.peek() == "%":
                operands.append(self.ssa()[0])
                while self.try_lit(","):
                    operands.append(self.ssa()[0])
                self.lit(":")
                self.ty()
                while self.try_lit(","):
                    self.ty()
            return L.Op(name, operands, [], {}, [], [], [])
        self.fail("unsupported op syntax %r (the generic form is expected)" % name)

    def skip_attrs(self) -> None:
        self.ws()
        if self.peek() == "{":
            self.attr_dict()

    def func(self) -> FuncDef:
        self.lit("func.func")
        self.try_lit("public")
        self.try_lit("private")
        self.lit("@")
        name = self.take_while(_id_char)
        self.lit("(")

        def arg():
            n = self.ssa()[0]
            self.lit(":")
            t = self.ty()
            self.skip_attrs()
            return n, t
        args = self.sep_by(arg, ")")
        outs = []
        if self.try_lit("->"):
            if self.try_lit("("):
                def out():
                    t = self.ty()
                    self.skip_attrs()
                    return t
                outs = self.sep_by(out, ")")
            else:
                outs = [self.ty()]
        if self.try_lit("attributes"):
            self.attr_dict()
        b = self.block()
        b.args = args
        return FuncDef(name, b, outs)

    def module(self) -> List[FuncDef]:
        wrapped = self.try_lit("module")
        if wrapped:
            if self.try_lit("@"):
                self.take_while(_id_char)
            if self.try_lit("attributes"):
                self.attr_dict()
            self.lit("{")
        fs = []
        while True:
            self.ws()
            if self.s.startswith("func.func", self.i):
                fs.append(self.func())
            else:
                break
        if wrapped:
            self.lit("}")
        self.ws()
        if self.peek() is not None:
            self.fail("trailing text after the module")
        return fs


def parse(text: str) -> List[FuncDef]:
    """Parse.lean:247."""
    return Reader(text).module()
