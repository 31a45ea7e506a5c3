"""The reference's kernel-grammar program IR, as plain data, plus a JSON form.

The reference describes every kernel it searches over as a ``Program`` of
``ParallelLoop`` stages whose bodies hold ``Load`` / ``Compute`` / ``Store``
statements and ``ReductionLoop`` s (``grammar/kernel_ast.py:27-99``).  The
B200 backend (``grammar_backend``) reads programs through exactly these class
names and fields, so it accepts the reference's own objects unchanged; the
dataclasses below let a caller (or a test) build the same programs without the
reference installed.  Field names and meanings follow the reference:

* ``Program(tensors, body)``            -- global shapes, list of stages
* ``ParallelLoop(out, tile_shape, index_vars, body)``
* ``Load(source, index)``               -- one axis name per dim of ``source``
* ``Compute(op, inputs, axis, const)``  -- ``op`` in matmul/add/sub/mul/div/
  relu/exp/sqrt/rowmax/rowsum/mulc/addc
* ``Store(dest, src, index)``
* ``ReductionLoop(axis, tile, body, partial, partials)``

``program_to_json`` / ``program_from_json`` keep node identity (a value used
twice is one node referenced twice) by numbering every node.
"""

from __future__ import annotations

from dataclasses import dataclass, field

Shape = tuple


@dataclass(eq=False)
class Program:
    tensors: dict
    body: list = field(default_factory=list)


@dataclass(eq=False)
class ParallelLoop:
    out: str
    tile_shape: tuple
    index_vars: tuple
    body: list = field(default_factory=list)


@dataclass(eq=False)
class Load:
    source: str
    index: list


@dataclass(eq=False)
class Compute:
    op: str
    inputs: list = field(default_factory=list)
    axis: str | None = None
    const: float | None = None


@dataclass(eq=False)
class Store:
    dest: str
    src: object
    index: list


@dataclass(eq=False)
class ReductionLoop:
    axis: str
    tile: int
    body: list = field(default_factory=list)
    partial: object = None
    partials: list | None = None

    def __post_init__(self):
        if self.partials is None:
            self.partials = [self.partial] if self.partial is not None else []
        if self.partial is None and self.partials:
            self.partial = self.partials[0]


def kind(node) -> str:
    """Class name of a node (works for the reference's classes and these)."""
    return type(node).__name__


# ---------------------------------------------------------------------------
# JSON form: {"tensors": {name: [dims]}, "body": [stage, ...], "nodes": [...]}
# Every Load / Compute / ReductionLoop / Store is a numbered entry of "nodes";
# bodies and operands refer to entries by number.
# ---------------------------------------------------------------------------
def program_to_json(program) -> dict:
    ids: dict[int, int] = {}
    nodes: list = []

    def ref(n) -> int:
        if id(n) in ids:
            return ids[id(n)]
        k = kind(n)
        slot = len(nodes)
        ids[id(n)] = slot
        nodes.append(None)
        if k == "Load":
            nodes[slot] = {"type": "Load", "source": n.source, "index": list(n.index)}
        elif k == "Compute":
            entry = {"type": "Compute", "op": n.op, "inputs": []}
            nodes[slot] = entry
            entry["inputs"] = [ref(i) for i in n.inputs]
            if n.axis is not None:
                entry["axis"] = n.axis
            if n.const is not None:
                entry["const"] = float(n.const)
        elif k == "Store":
            entry = {"type": "Store", "dest": n.dest, "index": list(n.index)}
            nodes[slot] = entry
            entry["src"] = ref(n.src)
        elif k == "ReductionLoop":
            entry = {"type": "ReductionLoop", "axis": n.axis, "tile": int(n.tile)}
            nodes[slot] = entry
            entry["body"] = [ref(s) for s in n.body]
            entry["partials"] = [ref(p) for p in (n.partials or [])]
        else:
            raise TypeError(f"unsupported node type {k}")
        return slot

    body = []
    for loop in program.body:
        if kind(loop) != "ParallelLoop":
            raise TypeError(f"program body holds {kind(loop)}, expected ParallelLoop")
        body.append({"out": loop.out, "tile_shape": list(loop.tile_shape),
                     "index_vars": list(loop.index_vars),
                     "body": [ref(s) for s in loop.body]})
    return {"tensors": {k: list(v) for k, v in program.tensors.items()}, "body": body,
            "nodes": nodes}


def program_from_json(obj: dict) -> Program:
    entries = obj["nodes"]
    built: dict[int, object] = {}

    def get(i: int):
        if i in built:
            return built[i]
        e = entries[i]
        t = e["type"]
        if t == "Load":
            n = Load(e["source"], list(e["index"]))
            built[i] = n
        elif t == "Compute":
            n = Compute(e["op"], [], e.get("axis"), e.get("const"))
            built[i] = n
            n.inputs = [get(j) for j in e["inputs"]]
        elif t == "Store":
            n = Store(e["dest"], None, list(e["index"]))
            built[i] = n
            n.src = get(e["src"])
        elif t == "ReductionLoop":
            n = ReductionLoop(e["axis"], e["tile"], [], None, [])
            built[i] = n
            n.body = [get(j) for j in e["body"]]
            n.partials = [get(j) for j in e["partials"]]
            n.partial = n.partials[0] if n.partials else None
        else:
            raise ValueError(f"unknown node type {t!r}")
        return n

    body = [ParallelLoop(s["out"], tuple(s["tile_shape"]), tuple(s["index_vars"]),
                         [get(j) for j in s["body"]]) for s in obj["body"]]
    return Program({k: tuple(v) for k, v in obj["tensors"].items()}, body)
